// qkv_tf32_sm100.cu -- the fused QKV projection: a layer's Q, K and V from its
// layer-normed input in ONE launch on the Blackwell tensor cores (sm_100a),
// fp32 in and out with 3xTF32 products.
//
// Semantics: the three gemm_nn calls of train_kaggle.cu:152-154,
//     Q = X Wq + bq,   K = X Wk + bk,   V = X Wv + bv
// with gemm_nn's conventions (gpu_kernels.cu:112-120: row-major fp32 C = A B,
// then the bias broadcast over rows, bias optional).  X is (M x Kd) with row
// stride ldx, each W is (Kd x N) row-major, and the outputs are (M x N) with
// row stride ldo -- three separate tensors, or the three column blocks of one
// (M x 3N) tensor that the attention kernels read as it is (in_row_stride 3N).
//
// Every product x*y is formed as xh*yh + xh*yl + xl*yh (xh: x with its 13 low
// mantissa bits cleared, exact in tf32; xl = x - xh, exact in fp32); the
// dropped xl*yl term is ~2^-21 relative.  The tensor core's accumulation into
// TMEM is not round-to-nearest, so a fresh TMEM sum starts every kFold k
// stages and the epilogue warps add the partial sums into fp32 registers.
//
// Persistent kernel, one 128 x 128 output tile per work item (the 3 * ceil(N/128)
// column tiles of the three outputs times ceil(M/128) row tiles), items dealt
// round-robin to one CTA per SM.  12 warps:
//   warp 0      TMA producer: X box (32 k x 128 rows) and W boxes (4 x 32 n x 32 k)
//               into a 3-stage ring
//   warp 1      MMA issuer: D += Xh Wh + Xh Wl + Xl Wh, M=128 N=128 K=8,
//               tcgen05.mma kind::tf32, into one of two TMEM accumulators
//   warps 2-3   idle
//   warps 4-7   splitters: X's high part in place and its low part beside it;
//               W transposed (K-major, as the B operand must be for tf32) as
//               high and low parts, by 4x4 micro-blocks
//   warps 8-11  epilogue: a thread owns one output row (one TMEM lane), adds
//               each partial sum into 128 fp32 registers, adds the bias and
//               writes the tile through shared memory with TMA stores
// Every mbarrier wait is bounded; a timeout records a code in the device
// error word, raises a CTA-wide abort flag, and all roles fall through to the
// teardown, which frees TMEM.
#include "common.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstdlib>

namespace attn {
namespace qkv {

using namespace sm100;

constexpr int BM = 128;            // output rows per tile (TMEM lanes)
constexpr int BN = 128;            // output columns per tile
constexpr int BK = 32;             // k per stage (one 128-byte swizzle row of fp32)
constexpr int kThreads = 384;
constexpr int kStages = 3;
constexpr int kFold = 8;           // k stages per fresh TMEM sum (256 k)
constexpr int XB = BM * BK * 4;    // 16 KB: one X part
constexpr int WB = BN * BK * 4;    // 16 KB: one W part
constexpr int STAGE = 2 * XB + 2 * WB;
constexpr int OFF_XH = 0, OFF_XL = XB, OFF_WL = 2 * XB, OFF_WH = 2 * XB + WB;   // within a stage
constexpr int OFF_OUT = kStages * STAGE;          // 4 epilogue warps x 2 buffers x 4 KB
constexpr int OFF_BAR = OFF_OUT + 4 * 2 * 4096;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr int TM_COLS = 2 * BN;                   // two accumulators
constexpr int REG_LOW = 72, REG_EPI = 232;        // 128 x (72 + 168 + 232) <= 384 x 168; no spills
static_assert(SMEM <= 227 * 1024, "shared memory");
static_assert(REG_LOW + 168 + REG_EPI <= 3 * 168, "register split exceeds the launch allocation");

enum {
    B_FULL = 0,                    // 3: stage landed
    B_SPLIT = 3,                   // 3: stage split
    B_EMPTY = 6,                   // 3: stage's MMAs finished
    B_ACCF = 9,                    // 2: accumulator holds a finished partial sum
    B_ACCE = 11,                   // 2: accumulator read by the epilogue
    B_SPL = 13,                    // splitters: raw W read (before W^T low overwrites it)
    B_COUNT = 14
};

struct Params {
    const float *bias[3];
    int M, N, K;
    int mt, nt;                    // row tiles, column tiles per output
    int n_items, nk;
    int *err;
};

__device__ __forceinline__ void item_coords(const Params &p, int item, int &m0, int &w, int &n0) {
    const int ng = item / p.mt;                    // consecutive CTAs share a column tile of W
    m0 = (item % p.mt) * BM;
    w = ng / p.nt;
    n0 = (ng % p.nt) * BN;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

__device__ __forceinline__ float f4_at(const float4 &v, int c) {
    return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
}
__device__ __forceinline__ float hi_part(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

__global__ void __launch_bounds__(kThreads, 1)
qkv_tf32_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tw0,
                const __grid_constant__ CUtensorMap tw1, const __grid_constant__ CUtensorMap tw2,
                const __grid_constant__ CUtensorMap to0, const __grid_constant__ CUtensorMap to1,
                const __grid_constant__ CUtensorMap to2, const __grid_constant__ Params p)
{
    pdl_begin();   // launched by launch_pdl
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *sb = smem_raw + (base - raw);
    const uint32_t bar0 = base + OFF_BAR;
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sb + OFF_BAR + 192);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sb + OFF_BAR + 196);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStages; i++) {
            mbar_init(BAR(B_FULL + i), 1);
            mbar_init(BAR(B_SPLIT + i), 128);
            mbar_init(BAR(B_EMPTY + i), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(BAR(B_ACCF + i), 1);
            mbar_init(BAR(B_ACCE + i), 128);
        }
        mbar_init(BAR(B_SPL), 128);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), TM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto wait_w = [&](int b, int parity, int code) -> bool {       // warp-wide bounded wait
        return __all_sync(0xffffffffu, mbar_wait(BAR(b), parity & 1, abort_flag, p.err, code));
    };

    if (warp < 8) {
        if (warp < 4) regs_dec<REG_LOW>();
        if (warp == 0) {
            // -------------------------------------------------------- producer
            const bool leader = elect_one();
            if (leader) {
                prefetch_tmap(&tx);
                prefetch_tmap(&tw0);
                prefetch_tmap(&tw1);
                prefetch_tmap(&tw2);
            }
            int g = 0;                                       // stages issued
            bool ok = true;
            for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
                int m0, w, n0;
                item_coords(p, item, m0, w, n0);
                const CUtensorMap *mw = w == 0 ? &tw0 : w == 1 ? &tw1 : &tw2;
                for (int ks = 0; ks < p.nk; ks++, g++) {
                    const int st = g % kStages;
                    if (g >= kStages && !(ok = wait_w(B_EMPTY + st, g / kStages - 1, 0x501))) break;
                    if (leader) {
                        const uint32_t s0 = base + st * STAGE;
                        mbar_arrive_expect_tx(BAR(B_FULL + st), XB + WB);
                        tma_load_2d(s0 + OFF_XH, &tx, BAR(B_FULL + st), ks * BK, m0);
#pragma unroll
                        for (int c = 0; c < BN / 32; c++)
                            tma_load_2d(s0 + OFF_WL + c * (BK * 128), mw, BAR(B_FULL + st), n0 + 32 * c, ks * BK);
                    }
                    __syncwarp();
                }
            }
        } else if (warp == 1) {
            // -------------------------------------------------------- MMA issuer
            const bool leader = elect_one();
            constexpr uint32_t idD = idesc_tf32(BM, BN, 0, 0);      // X, W^T both K-major
            int g = 0, ch = 0;
            bool ok = true;
            for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
                for (int ks = 0; ks < p.nk; ks++, g++) {
                    const int a = ch & 1;
                    if (ks % kFold == 0 && ch >= 2 && !(ok = wait_w(B_ACCE + a, ch / 2 - 1, 0x511))) break;
                    const int st = g % kStages;
                    if (!(ok = wait_w(B_SPLIT + st, g / kStages, 0x512))) break;
                    tc_fence_after();
                    const uint32_t s0 = base + st * STAGE;
                    if (leader) {
#pragma unroll
                        for (int part = 0; part < 3; part++) {       // hh, hl, lh
                            const uint32_t xa = s0 + (part == 2 ? OFF_XL : OFF_XH);
                            const uint32_t wb = s0 + (part == 1 ? OFF_WL : OFF_WH);
#pragma unroll
                            for (int kk = 0; kk < BK / 8; kk++)
                                mma_tf32_ss(tmem + BN * a, sw128_desc(xa + 32 * kk, 16, 1024),
                                            sw128_desc(wb + 32 * kk, 16, 1024), idD,
                                            (ks % kFold > 0 || part > 0 || kk > 0));
                        }
                        mma_commit(BAR(B_EMPTY + st));
                    }
                    const bool last = ks % kFold == kFold - 1 || ks == p.nk - 1;
                    if (last) {
                        if (leader) mma_commit(BAR(B_ACCF + a));
                        ch++;
                    }
                    __syncwarp();
                }
            }
        } else if (warp >= 4) {
            // -------------------------------------------------------- splitters
            const int tid = threadIdx.x - 128;
            int g = 0;
            bool ok = true;
            for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
                for (int ks = 0; ks < p.nk; ks++, g++) {
                    const int st = g % kStages;
                    if (!(ok = wait_w(B_FULL + st, g / kStages, 0x521))) break;
                    uint8_t *s0 = sb + st * STAGE;
                    // X: high part in place, low part beside it (same swizzled offsets)
                    {
                        float *xh = reinterpret_cast<float *>(s0 + OFF_XH);
                        float *xl = reinterpret_cast<float *>(s0 + OFF_XL);
#pragma unroll
                        for (int i = 0; i < BM * BK / (128 * 4); i++) {
                            const int e = 4 * (tid + 128 * i);
                            const float4 x = *reinterpret_cast<const float4 *>(xh + e);
                            const float4 h = make_float4(hi_part(x.x), hi_part(x.y), hi_part(x.z), hi_part(x.w));
                            *reinterpret_cast<float4 *>(xh + e) = h;
                            *reinterpret_cast<float4 *>(xl + e) = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
                        }
                    }
                    // W: raw boxes ([32 k][32 n] per 32-column chunk, 128-byte swizzle)
                    // -> W^T high and low ([128 n][32 k], K-major, same swizzle).  4x4
                    // micro-blocks with 16-byte loads and stores; the 8 lanes of each
                    // quarter-warp take one diagonal of a 32 x 32 block's 8 x 8 grid of
                    // micro-blocks (k group a, n group b = a + p mod 8), so their loads
                    // hit 8 different 16-byte bank groups, and so do their stores.
                    // Every raw value is read before the low part overwrites the raw tile.
                    uint8_t *wraw = s0 + OFF_WL;
                    constexpr int MB = BN * BK / 16 / 128;     // micro-blocks per thread
                    float4 vr[MB][4];
#pragma unroll
                    for (int u = 0; u < MB; u++) {
                        const int m = tid + 128 * u, c32 = m >> 6, a = m & 7, b = (a + ((m & 63) >> 3)) & 7;
#pragma unroll
                        for (int r = 0; r < 4; r++) {
                            const int k = 4 * a + r;
                            vr[u][r] = *reinterpret_cast<const float4 *>(wraw + c32 * (BK * 128) + k * 128 +
                                                                         ((b ^ (k & 7)) << 4));
                        }
                    }
                    mbar_arrive(BAR(B_SPL));
                    if (!(ok = wait_w(B_SPL, g, 0x522))) break;
#pragma unroll
                    for (int u = 0; u < MB; u++) {
                        const int m = tid + 128 * u, c32 = m >> 6, a = m & 7, b = (a + ((m & 63) >> 3)) & 7;
#pragma unroll
                        for (int c = 0; c < 4; c++) {
                            const int n = 32 * c32 + 4 * b + c;
                            const int off = n * 128 + ((a ^ (n & 7)) << 4);
                            const float x[4] = {f4_at(vr[u][0], c), f4_at(vr[u][1], c), f4_at(vr[u][2], c),
                                                f4_at(vr[u][3], c)};
                            float h[4], l[4];
#pragma unroll
                            for (int r = 0; r < 4; r++) {
                                h[r] = hi_part(x[r]);
                                l[r] = x[r] - h[r];
                            }
                            *reinterpret_cast<float4 *>(s0 + OFF_WH + off) = make_float4(h[0], h[1], h[2], h[3]);
                            *reinterpret_cast<float4 *>(wraw + off) = make_float4(l[0], l[1], l[2], l[3]);
                        }
                    }
                    fence_async_smem();
                    mbar_arrive(BAR(B_SPLIT + st));
                }
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        regs_inc<REG_EPI>();
        const int quad = warp & 3;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        uint8_t *stage_out = sb + OFF_OUT + quad * 8192;
        const bool leader = lane == 0;
        const int nchunks = (p.nk + kFold - 1) / kFold;
        float acc[BN];
        int ch = 0;
        bool ok = true;
        for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
            int m0, w, n0;
            item_coords(p, item, m0, w, n0);
#pragma unroll
            for (int c = 0; c < BN; c++) acc[c] = 0.f;
            for (int c = 0; c < nchunks; c++, ch++) {
                const int a = ch & 1;
                if (!(ok = wait_w(B_ACCF + a, ch / 2, 0x531))) break;
                tc_fence_after();
#pragma unroll
                for (int q = 0; q < BN / 16; q++) {
                    uint32_t r[16];
                    tmem_ld16(tmem + lane_base + BN * a + 16 * q, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; i++) acc[16 * q + i] += __uint_as_float(r[i]);
                }
                tc_fence_before();
                mbar_arrive(BAR(B_ACCE + a));
            }
            if (!ok) break;
            // bias, then 32 x 32 blocks through shared memory (128-byte swizzle) to TMA stores
            const float *bias = p.bias[w];
            const CUtensorMap *mo = w == 0 ? &to0 : w == 1 ? &to1 : &to2;
            const bool rows_in = m0 + 32 * quad < p.M;       // TMA clips partial boxes; skip empty ones
#pragma unroll
            for (int q = 0; q < BN / 32; q++) {
                const int col0 = n0 + 32 * q;
                if (col0 >= p.N || !rows_in) break;
                float *v = acc + 32 * q;
                if (bias) {
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (col0 + i < p.N) v[i] += __ldg(bias + col0 + i);
                }
                if (leader) bulk_wait_read_1();              // this buffer's previous store has read it
                __syncwarp();
                uint8_t *buf = stage_out + (q & 1) * 4096;
#pragma unroll
                for (int j = 0; j < 8; j++)
                    *reinterpret_cast<float4 *>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                fence_async_smem();
                __syncwarp();
                if (leader) {
                    tma_store_2d(mo, smem_u32(buf), col0, m0 + 32 * quad);
                    bulk_commit_group();
                }
            }
        }
        if (leader) bulk_wait_all();
        __syncwarp();
    }

    // ---------------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        for (int i = 0; i < 1000; i++) __nanosleep(1000);
    }
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, TM_COLS);
    }
#undef BAR
}

}  // namespace qkv
}  // namespace attn

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace attn_host {

bool ensure_smem_attr(const void *func, size_t bytes);
int sm_count_here();
bool ensure_carveout(const void *func, int percent);

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn_qkv() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// 2-D view {cols, rows} of a row-major fp32 matrix, `box_cols` x `box_rows`
// boxes with the 128-byte swizzle.
static bool map_2d(CUtensorMap *m, const void *ptr, long long cols, long long rows, long long stride, int box_cols,
                   int box_rows) {
    auto fn = encode_fn_qkv();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)stride * 4};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_qkv_tf32_sm100(const attn_qkv_shape *s, const float *x, const float *const w[3],
                          const float *const bias[3], float *const out[3], int *err, cudaStream_t stream) {
    using namespace attn::qkv;
    const long long ldx = s->x_row_stride ? s->x_row_stride : s->in_features;
    const long long ldo = s->out_row_stride ? s->out_row_stride : s->out_features;
    CUtensorMap mx, mw[3], mo[3];
    if (!map_2d(&mx, x, s->in_features, s->rows, ldx, BK, BM))
        return set_error(ATTN_ERR_CUDA, "QKV projection: cuTensorMapEncodeTiled failed (X)");
    for (int i = 0; i < 3; i++)
        if (!map_2d(&mw[i], w[i], s->out_features, s->in_features, s->out_features, 32, BK) ||
            !map_2d(&mo[i], out[i], s->out_features, s->rows, ldo, 32, 32))
            return set_error(ATTN_ERR_CUDA, "QKV projection: cuTensorMapEncodeTiled failed (W or output)");
    Params p;
    for (int i = 0; i < 3; i++) p.bias[i] = bias[i];
    p.M = s->rows;
    p.N = s->out_features;
    p.K = s->in_features;
    p.mt = (p.M + BM - 1) / BM;
    p.nt = (p.N + BN - 1) / BN;
    p.n_items = 3 * p.mt * p.nt;
    p.nk = (p.K + BK - 1) / BK;
    p.err = err;
    const int ctas = std::max(1, std::min(sm_count_here(), p.n_items));
    if (!ensure_smem_attr((const void *)qkv_tf32_kernel, SMEM))
        return set_error(ATTN_ERR_CUDA, "QKV projection: cannot set shared-memory size");
    if (!ensure_carveout((const void *)qkv_tf32_kernel, 100))
        return set_error(ATTN_ERR_CUDA, "QKV projection: cannot set the shared-memory carveout");
    return check_pdl(launch_pdl(qkv_tf32_kernel, dim3(ctas), dim3(kThreads), (size_t)SMEM, stream, mx, mw[0], mw[1],
                                mw[2], mo[0], mo[1], mo[2], p),
                     "QKV projection kernel");
}

}  // namespace attn_host

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
namespace attn_host {
int *device_error_ptr();
}

extern "C" {

int attn_qkv_proj_ex(const attn_qkv_shape *s, const float *x, const float *wq, const float *wk, const float *wv,
                     const float *bq, const float *bk, const float *bv, float *q, float *k, float *v,
                     attn_stream_t stream) {
    using attn_host::set_error;
    if (!s) return set_error(ATTN_ERR_INVALID, "QKV projection: shape is NULL");
    if (s->rows < 0 || s->in_features < 1 || s->out_features < 1)
        return set_error(ATTN_ERR_INVALID, "QKV projection: bad shape rows=%d in=%d out=%d", s->rows,
                         s->in_features, s->out_features);
    if (s->rows == 0) return ATTN_OK;
    const long long ldx = s->x_row_stride ? s->x_row_stride : s->in_features;
    const long long ldo = s->out_row_stride ? s->out_row_stride : s->out_features;
    if (ldx < s->in_features || ldo < s->out_features || ldx % 4 || ldo % 4 || s->out_features % 4)
        return set_error(ATTN_ERR_INVALID,
                         "QKV projection: out_features (%d) and the row strides (%lld, %lld) must be multiples "
                         "of 4, strides >= the row lengths", s->out_features, ldx, ldo);
    const void *ptrs[7] = {x, wq, wk, wv, q, k, v};
    for (const void *ptr : ptrs) {
        if (!ptr) return set_error(ATTN_ERR_INVALID, "QKV projection: NULL tensor pointer");
        if (reinterpret_cast<uintptr_t>(ptr) & 15)
            return set_error(ATTN_ERR_INVALID, "QKV projection: tensors must be 16-byte aligned");
    }
    const float *w[3] = {wq, wk, wv};
    const float *b[3] = {bq, bk, bv};
    float *o[3] = {q, k, v};
    return attn_host::launch_qkv_tf32_sm100(s, x, w, b, o, attn_host::device_error_ptr(),
                                            reinterpret_cast<cudaStream_t>(stream));
}

void attn_qkv_proj(const float *X, const float *Wq, const float *Wk, const float *Wv, const float *bq,
                   const float *bk, const float *bv, float *Q, float *K, float *V, int M, int K_, int N) {
    const attn_qkv_shape s = {M, K_, N, 0, 0};
    const int st = attn_qkv_proj_ex(&s, X, Wq, Wk, Wv, bq, bk, bv, Q, K, V, nullptr);
    if (st != ATTN_OK) {
        fprintf(stderr, "CUDA error '%s' at attn_qkv_proj\n", attn_last_error());
        exit(1);
    }
}

}  // extern "C"
