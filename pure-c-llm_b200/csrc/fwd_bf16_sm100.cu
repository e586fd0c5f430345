// fwd_bf16_sm100.cu -- causal flash forward on the Blackwell tensor cores.
//
// Semantics: attention_forward, train.c:339-370, with bf16 Q/K/V/O and fp32
// scores, softmax statistics and accumulators (the tolerance of this path is
// stated against fp32 attention over the same bf16 inputs).
//
// One CTA per (pair of 128-row query tiles, head, batch), 12 warps:
//   warp 0      TMA producer: Q tiles once, then K_j/V_j into a 4-stage ring
//   warp 1      MMA issuer (one thread): S_i = Q_i K_j^T (both operands in
//               shared memory) and O_i += P_i V_j (P from TMEM, V from shared
//               memory) with tcgen05.mma kind::f16, accumulators in TMEM
//   warps 4-7   softmax for query tile 0; warps 8-11 for query tile 1.  A
//               thread owns one query row (= one TMEM lane): it reads its S
//               row with tcgen05.ld, keeps the running max/sum, writes its
//               row of P (bf16 pairs) back into TMEM with tcgen05.st, and
//               rescales its O row in TMEM when the max grew by more than 2^8
//               (otherwise the stale max is kept; the final normalisation uses
//               the same max for O and the sum).
// The two query tiles ping-pong: while one warpgroup runs softmax, the
// tensor core works on the other tile's products.  Keeping P in TMEM halves
// the shared-memory traffic of the PV product (which would otherwise read
// 6 KB per 32 tensor cycles, above the ~128 B/clk shared-memory bandwidth).
//
// TMEM: S0 cols [0,128), S1 [128,256), O0 [256,256+D), O1 [256+D, 256+2D),
// P0 and P1 64 columns each after the O tiles.
// Every mbarrier wait is bounded; a timeout records a code in the device
// error word, raises a CTA-wide abort flag, and all roles fall through to the
// common teardown, which frees TMEM.
#include "common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

namespace attn {
namespace fa {

using namespace sm100;

constexpr int BM = 128;           // query rows per tile (TMEM lanes)
constexpr int BN = 128;           // keys per tile
constexpr int kStages = 4;
constexpr int kThreads = 384;

template <int D>
struct Cfg {
    static constexpr int Q_BYTES = BM * D * 2;
    static constexpr int KV_BYTES = BN * D * 2;
    static constexpr int OFF_Q = 0;
    static constexpr int OFF_KV = 2 * Q_BYTES;
    static constexpr int STAGE_BYTES = 2 * KV_BYTES;
    static constexpr int OFF_BAR = OFF_KV + kStages * STAGE_BYTES;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;
    // TMEM columns: S (fp32, 128 keys) and O (fp32, D) per query tile, and P
    // (bf16 pairs, 64 columns for 128 keys) per query tile
    static constexpr int TM_S0 = 0, TM_S1 = 128, TM_O0 = 256, TM_O1 = 256 + D;
    static constexpr int TM_P0 = 256 + 2 * D, TM_P1 = 256 + 2 * D + BN / 2;
    static constexpr int TM_COLS = 512;
    static_assert(TM_P1 + BN / 2 <= TM_COLS, "TMEM budget");
};

// barrier slots
enum { B_Q = 0, B_KVF = 1, B_KVE = 1 + kStages, B_SF = 1 + 2 * kStages, B_SE = B_SF + 2, B_PF = B_SE + 2,
       B_OD = B_PF + 2, B_COUNT = B_OD + 2 };

struct Params {
    __nv_bfloat16 *o;
    float *lse;
    long long out_stride;
    int T, H, n_pairs;
    float scale_log2;     // log2(e) / sqrt(d)
    int *err;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
           const __grid_constant__ CUtensorMap tv, const Params p)
{
    using C = Cfg<D>;
    static_assert(D == 64, "this kernel instance covers head_dim 64");
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *sb = smem_raw + (base - raw);
    const uint32_t sQ = base + C::OFF_Q, sKV = base + C::OFF_KV;
    const uint32_t bar0 = base + C::OFF_BAR;
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sb + C::OFF_BAR + 128);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sb + C::OFF_BAR + 132);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the pair index is the slowest grid dimension, so every CTA of the
    // heaviest pairs (most key tiles) is issued before any lighter one
    const int pair = p.n_pairs - 1 - (int)blockIdx.z;
    const int h = blockIdx.x, b = blockIdx.y;
    const int q0 = pair * 2 * BM;
    const bool has_q1 = (q0 + BM) < p.T;
    const int n0 = q0 / BN + 1;                  // key tiles of query tile 0 (last is diagonal)
    const int n1 = has_q1 ? n0 + 1 : 0;          // key tiles of query tile 1
    const int n_kv = has_q1 ? n1 : n0;           // key tiles streamed by this CTA

    if (threadIdx.x == 0) {
        mbar_init(BAR(B_Q), 1);
        for (int s = 0; s < kStages; s++) { mbar_init(BAR(B_KVF + s), 1); mbar_init(BAR(B_KVE + s), 1); }
        for (int i = 0; i < 2; i++) {
            mbar_init(BAR(B_SF + i), 1);
            mbar_init(BAR(B_SE + i), 128);
            mbar_init(BAR(B_PF + i), 128);
            mbar_init(BAR(B_OD + i), 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_u32(tmem_slot), C::TM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // registers: 384 x 168 at launch; warpgroup 0 (TMA, MMA, 2 spare warps)
    // gives back down to 72 so the two softmax warpgroups can hold 216 each
    // (128 x 72 + 256 x 216 = 384 x 168).  Each setmaxnreg sits inside its
    // role's branch so that it dominates the code that uses the new budget.
    if (warp < 4) regs_dec<72>();
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tmap(&tq);
            prefetch_tmap(&tk);
            prefetch_tmap(&tv);
            mbar_arrive_expect_tx(BAR(B_Q), (has_q1 ? 2 : 1) * C::Q_BYTES);
            tma_load_3d(sQ, &tq, BAR(B_Q), h * D, q0, b);
            if (has_q1) tma_load_3d(sQ + C::Q_BYTES, &tq, BAR(B_Q), h * D, q0 + BM, b);
            for (int j = 0; j < n_kv; j++) {
                const int st = j % kStages;
                if (j >= kStages &&
                    !mbar_wait(BAR(B_KVE + st), ((j / kStages) + 1) & 1, abort_flag, p.err, 0x201))
                    break;
                mbar_arrive_expect_tx(BAR(B_KVF + st), 2 * C::KV_BYTES);
                const uint32_t dst = sKV + st * C::STAGE_BYTES;
                tma_load_3d(dst, &tk, BAR(B_KVF + st), h * D, j * BN, b);
                tma_load_3d(dst + C::KV_BYTES, &tv, BAR(B_KVF + st), h * D, j * BN, b);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idS = idesc_bf16(BM, BN, 0, 0);   // Q, K both K-major
            constexpr uint32_t idO = idesc_bf16(BM, D, 0, 1);    // P K-major, V MN-major
            auto issue_S = [&](int i, int j) {
                const uint32_t ka = sKV + (j % kStages) * C::STAGE_BYTES;
                const uint32_t qa = sQ + i * C::Q_BYTES;
                const uint32_t d_t = tmem + (i ? C::TM_S1 : C::TM_S0);
#pragma unroll
                for (int kk = 0; kk < D / 16; kk++)
                    mma_bf16_ss(d_t, sw128_desc(qa + kk * 32, 16, 1024), sw128_desc(ka + kk * 32, 16, 1024), idS,
                                kk > 0);
                mma_commit(BAR(B_SF + i));
            };
            auto issue_PV = [&](int i, int j) {
                const uint32_t va = sKV + (j % kStages) * C::STAGE_BYTES + C::KV_BYTES;
                const uint32_t pt = tmem + (i ? C::TM_P1 : C::TM_P0);
                const uint32_t d_t = tmem + (i ? C::TM_O1 : C::TM_O0);
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++)      // 16 keys = 8 packed TMEM columns per step
                    mma_bf16_ts(d_t, pt + kk * 8, sw128_desc(va + kk * 16 * 128, 16384, 1024), idO,
                                (j > 0 || kk > 0));
                mma_commit(BAR(B_OD + i));
            };
            bool ok = mbar_wait(BAR(B_Q), 0, abort_flag, p.err, 0x211) &&
                      mbar_wait(BAR(B_KVF + 0), 0, abort_flag, p.err, 0x212);
            if (ok) {
                tc_fence_after();
                issue_S(0, 0);
                if (has_q1) issue_S(1, 0);
            }
            // Per key tile j: the scores of tile j+1 are issued as soon as each
            // warpgroup has drained its S buffer (it does so right after loading
            // S_j, before its softmax), so S_{j+1} is ready by the time P_j is;
            // the PV products of tile j follow when P_j arrives.  A warpgroup
            // therefore never waits for its own MMAs between tiles.
            for (int j = 0; ok && j < n_kv; j++) {
                const int nx = j + 1, nst = nx % kStages;
                const bool s0_next = nx < n0, s1_next = has_q1 && nx < n1;
                if (s0_next || s1_next) {
                    if (!(ok = mbar_wait(BAR(B_KVF + nst), (nx / kStages) & 1, abort_flag, p.err, 0x214))) break;
                }
                if (s0_next) {
                    if (!(ok = mbar_wait(BAR(B_SE + 0), j & 1, abort_flag, p.err, 0x215))) break;
                    tc_fence_after();
                    issue_S(0, nx);
                }
                if (s1_next) {
                    if (!(ok = mbar_wait(BAR(B_SE + 1), j & 1, abort_flag, p.err, 0x218))) break;
                    tc_fence_after();
                    issue_S(1, nx);
                }
                if (j < n0) {
                    if (!(ok = mbar_wait(BAR(B_PF + 0), j & 1, abort_flag, p.err, 0x213))) break;
                    tc_fence_after();
                    issue_PV(0, j);
                }
                if (has_q1) {
                    if (!(ok = mbar_wait(BAR(B_PF + 1), j & 1, abort_flag, p.err, 0x216))) break;
                    tc_fence_after();
                    issue_PV(1, j);
                }
                mma_commit(BAR(B_KVE + j % kStages));      // stage j free once these MMAs finish
            }
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ softmax
        regs_inc<216>();
        const int wg = (warp - 4) >> 2;
        const int quad = warp & 3;                   // TMEM lane quadrant of this warp
        const int row = quad * 32 + lane;            // query row within the tile
        const int n = wg ? n1 : n0;
        const int qs = q0 + wg * BM;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const uint32_t tS = tmem + lane_base + (wg ? C::TM_S1 : C::TM_S0);
        const uint32_t tO = tmem + lane_base + (wg ? C::TM_O1 : C::TM_O0);
        const uint32_t tP = tmem + lane_base + (wg ? C::TM_P1 : C::TM_P0);
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < n; j++) {
            ok = mbar_wait(BAR(B_SF + wg), j & 1, abort_flag, p.err, 0x221);
            if (!(ok = __all_sync(0xffffffffu, ok))) break;   // tcgen05.ld below is warp-collective
            tc_fence_after();
            uint32_t s[128];
#pragma unroll
            for (int q4 = 0; q4 < 4; q4++) {         // (copies keep `s` in registers)
                uint32_t t[32];
                tmem_ld32(tS + 32 * q4, t);
#pragma unroll
                for (int c = 0; c < 32; c++) s[32 * q4 + c] = t[c];
            }
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(BAR(B_SE + wg));             // S buffer may be overwritten now

            // row max as 8 independent partial chains (a single 128-long chain of
            // dependent max operations would serialise on instruction latency)
            float mp[8];
#pragma unroll
            for (int i = 0; i < 8; i++) mp[i] = -INFINITY;
            if (j == n - 1) {                        // diagonal tile: keys past the query row are masked
#pragma unroll
                for (int c = 0; c < 128; c++) {
                    const float v = c > row ? -INFINITY : __uint_as_float(s[c]);
                    s[c] = __float_as_uint(v);
                    mp[c & 7] = fmaxf(mp[c & 7], v);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 128; c++) mp[c & 7] = fmaxf(mp[c & 7], __uint_as_float(s[c]));
            }
            float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
            mx *= p.scale_log2;
            float alpha = 1.f;
            const bool grow = mx > m_run + 8.f;      // also true on the first tile
            if (grow) {
                alpha = ex2(m_run - mx);
                m_run = mx;
                l_run *= alpha;
            }
            const float neg_m = -m_run;
            float lp[8];
#pragma unroll
            for (int i = 0; i < 8; i++) lp[i] = 0.f;
#pragma unroll
            for (int c = 0; c < 128; c++) {
                const float e = ex2(fmaf(__uint_as_float(s[c]), p.scale_log2, neg_m));
                s[c] = __float_as_uint(e);
                lp[c & 7] += e;
            }
            l_run += ((lp[0] + lp[1]) + (lp[2] + lp[3])) + ((lp[4] + lp[5]) + (lp[6] + lp[7]));
            // P buffer and O are in use by the previous PV until it completes
            if (j > 0) ok = mbar_wait(BAR(B_OD + wg), (j - 1) & 1, abort_flag, p.err, 0x222);
            if (!(ok = __all_sync(0xffffffffu, ok))) break;
            tc_fence_after();
            // P row -> TMEM as bf16 pairs (keys 2c, 2c+1 in column c): the A
            // operand of the next PV product
#pragma unroll
            for (int half = 0; half < 2; half++) {
                uint32_t t[32];
#pragma unroll
                for (int c = 0; c < 32; c++)
                    t[c] = pack_bf16(__uint_as_float(s[64 * half + 2 * c]), __uint_as_float(s[64 * half + 2 * c + 1]));
                tmem_st32(tP + 32 * half, t);
            }
            // rows whose max did not grow keep alpha = 1; the TMEM round trip is
            // warp-collective, so a warp rescales if any of its rows needs it
            if (__any_sync(0xffffffffu, j > 0 && grow)) {
                uint32_t o[32];
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 32) {
                    tmem_ld32(tO + c0, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; c++) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                    tmem_st32(tO + c0, o);
                }
            }
            tmem_wait_st();                          // P (and O) stores complete before the MMA reads them
            tc_fence_before();
            mbar_arrive(BAR(B_PF + wg));
        }
        if (ok && n > 0) ok = mbar_wait(BAR(B_OD + wg), (n - 1) & 1, abort_flag, p.err, 0x223);
        if (__all_sync(0xffffffffu, ok && n > 0)) {
            tc_fence_after();
            const int qrow = qs + row;
            const float inv = 1.f / l_run;
            uint32_t o[32];
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += 32) {
                tmem_ld32(tO + c0, o);
                tmem_wait_ld();
                if (qrow < p.T) {
                    __nv_bfloat16 *dst = p.o + ((long long)b * p.T + qrow) * p.out_stride + (long long)h * D + c0;
#pragma unroll
                    for (int c = 0; c < 32; c += 8) {
                        uint4 v;
                        v.x = pack_bf16(__uint_as_float(o[c + 0]) * inv, __uint_as_float(o[c + 1]) * inv);
                        v.y = pack_bf16(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
                        v.z = pack_bf16(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv);
                        v.w = pack_bf16(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv);
                        *reinterpret_cast<uint4 *>(dst + c) = v;
                    }
                }
            }
            if (p.lse && qrow < p.T)
                p.lse[((long long)b * p.H + h) * p.T + qrow] = (m_run + __log2f(l_run)) * kLn2;
        }
    }

    // ---------------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        // let copies / MMAs already in flight drain before the CTA releases its memory
        for (int i = 0; i < 1000; i++) __nanosleep(1000);
    }
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TM_COLS);
    }
#undef BAR
}

}  // namespace fa
}  // namespace attn

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace attn_host {

bool ensure_smem_attr(const void *func, size_t bytes);

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 3-D view {columns, T, B} of a (B*T, stride) bf16 activation; 64 x 128 boxes
// with the 128-byte swizzle the MMA descriptors expect.
static bool make_map(CUtensorMap *m, const void *ptr, int cols, int T, int B, long long stride) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)stride * 2, (cuuint64_t)stride * 2 * T};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool fwd_bf16_sm100_supported(int D, long long in_stride, long long out_stride) {
    return D == 64 && in_stride % 8 == 0 && out_stride % 8 == 0 && encode_fn() != nullptr;
}

int launch_fwd_bf16_sm100(int D, const void *q, const void *k, const void *v, void *o, float *lse,
                          long long in_stride, long long out_stride, int B, int H, int T, int *err,
                          cudaStream_t s) {
    using namespace attn::fa;
    if (D != 64) return set_error(ATTN_ERR_UNSUPPORTED, "tcgen05 forward: head_dim %d", D);
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15)
        return set_error(ATTN_ERR_INVALID, "tcgen05 forward: tensors must be 16-byte aligned");
    CUtensorMap tq, tk, tv;
    if (!make_map(&tq, q, H * D, T, B, in_stride) || !make_map(&tk, k, H * D, T, B, in_stride) ||
        !make_map(&tv, v, H * D, T, B, in_stride))
        return set_error(ATTN_ERR_CUDA, "tcgen05 forward: cuTensorMapEncodeTiled failed");
    Params p;
    p.o = static_cast<__nv_bfloat16 *>(o);
    p.lse = lse;
    p.out_stride = out_stride;
    p.T = T;
    p.H = H;
    p.n_pairs = (T + 2 * BM - 1) / (2 * BM);
    p.scale_log2 = attn::kLog2e / sqrtf((float)D);
    p.err = err;
    const size_t smem = Cfg<64>::SMEM;
    if (!ensure_smem_attr((const void *)fwd_kernel<64>, smem))
        return set_error(ATTN_ERR_CUDA, "tcgen05 forward: cannot set shared-memory size");
    dim3 grid(H, B, p.n_pairs);
    fwd_kernel<64><<<grid, kThreads, smem, s>>>(tq, tk, tv, p);
    return check_launch("tcgen05 forward kernel");
}

}  // namespace attn_host
