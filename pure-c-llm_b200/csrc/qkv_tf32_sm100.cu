// qkv_tf32_sm100.cu -- fp32 GEMMs on the Blackwell tensor cores (sm_100a) with
// 3xTF32 products: the fused QKV projection (a layer's Q, K and V from its
// layer-normed input in ONE launch), and -- the same kernel in three more
// modes (see Params) -- the causal attention backward at head dims 96 and 128
// as GEMMs over explicit score tiles (launch_bwd_tc, the attn_bwd drop-in's
// path; attention_backward, train.c:373-407).
//
// Semantics: the three gemm_nn calls of train_kaggle.cu:152-154,
//     Q = X Wq + bq,   K = X Wk + bk,   V = X Wv + bv
// with gemm_nn's conventions (gpu_kernels.cu:112-120: row-major fp32 C = A B,
// then the bias broadcast over rows, bias optional).  X is (M x Kd) with row
// stride ldx, each W is (Kd x N) row-major, and the outputs are (M x N) with
// row stride ldo -- three separate tensors, or the three column blocks of one
// (M x 3N) tensor that the attention kernels read as it is (in_row_stride 3N).
//
// Every product x*y is formed as xh*yh + xh*yl + xl*yh (xh: x rounded to the
// nearest tf32 value, exact in tf32; xl = x - xh, exact in fp32); the
// dropped xl*yl term is ~2^-22 relative.  The tensor core's accumulation into
// TMEM is not round-to-nearest, so a fresh TMEM sum starts every Params::fold k
// stages and the epilogue warps add the partial sums into fp32 registers.
//
// Two launches per call:
//   qkv_split_w_kernel  the three weights, transposed to (N x K) rows (K-major,
//               as the tf32 B operand must be) and split into high and low parts,
//               into a workspace [part][3N][Kp] (Kp = K rounded up to 4); every
//               weight element is read once and written twice, instead of being
//               re-split by each of the ceil(M/128) row tiles that use it
//   qkv_tf32_kernel  persistent, one 128 x 128 output tile per work item (the
//               3 * ceil(N/128) column tiles of the three outputs times ceil(M/128)
//               row tiles), items dealt round-robin to one CTA per SM.  12 warps:
//   warp 0      TMA producer: per 32-k stage the raw X box (32 k x 128 rows) and
//               the W^T high and low boxes (32 k x 128 n) into a 4-stage ring
//   warp 1      MMA issuer: D += Xh Wh + Xh Wl + Xl Wh, M=128 N=128 K=8,
//               tcgen05.mma kind::tf32 with A (X's parts) from TMEM and B from
//               shared memory, into one of two TMEM accumulators
//   warps 2-3   idle
//   warps 4-7   splitters: X's high and low parts into the stage's TMEM slot (a
//               warp per 32 rows, its TMEM lane quadrant)
//   warps 8-11  epilogue: a thread owns one output row (one TMEM lane), adds
//               each partial sum into 128 fp32 registers, adds the bias and
//               writes the tile through shared memory with TMA stores
// Shared memory's 128 bytes per clock bound this kernel: with both operands
// in shared memory and both split there, a 32-k stage moved 224 KB through it
// against ~770 cycles of tensor work.  Now a stage moves 112 KB: TMA's 48 KB,
// the splitters' 16 KB read of X, and the MMAs' 48 KB read of W's parts.
// Every mbarrier wait is bounded; a timeout records a code in the device
// error word, raises a CTA-wide abort flag, and all roles fall through to the
// teardown, which frees TMEM.
#include "common.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <atomic>
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

namespace attn {
namespace qkv {

using namespace sm100;

constexpr int BM = 128;            // output rows per tile (TMEM lanes)
constexpr int BN = 128;            // output columns per tile
constexpr int BK = 32;             // k per stage (one 128-byte swizzle row of fp32)
constexpr int kThreads = 384;
constexpr int kStages = 4;
// k stages per fresh TMEM sum (Params::fold): 8 (256 k) for the projection;
// 2 (64 k) for the backward's GEMMs, whose sums cancel more: at the trainer
// shape their largest errors against the reference fall from 3.4e-6 (dQ),
// 6.5e-6 (dK) and 5.1e-6 (dV) with 8 to 1.6e-6, 3.3e-6 and 2.7e-6, for 1 % of
// the backward's time (1 stage: 1.0e-6 / 2.5e-6 / 2.2e-6, 7 % slower).
constexpr int kFoldQKV = 8, kFoldBwd = 2;
constexpr int XB = BM * BK * 4;    // 16 KB: one X part
constexpr int WB = BN * BK * 4;    // 16 KB: one W part
constexpr int STAGE = XB + 2 * WB;
constexpr int OFF_X = 0, OFF_WH = XB, OFF_WL = XB + WB;   // within a stage: raw X, W^T high, W^T low
constexpr int OFF_OUT = kStages * STAGE;          // 4 epilogue warps x 2 buffers x 4 KB
constexpr int OFF_BAR = OFF_OUT + 4 * 2 * 4096;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr int TM_X = 2 * BN;                      // TMEM: two accumulators, then per stage Xh, Xl (32 each)
constexpr int TM_COLS = 512;
static_assert(TM_X + 64 * kStages <= TM_COLS, "TMEM budget");
constexpr int REG_LOW = 104, REG_EPI = 232;       // 128 x (104 + 168 + 232) <= 384 x 168; no spills
static_assert(SMEM <= 227 * 1024, "shared memory");
static_assert(REG_LOW + 168 + REG_EPI <= 3 * 168, "register split exceeds the launch allocation");

enum {
    B_FULL = 0,                    // 4: stage landed
    B_SPLIT = 4,                   // 4: stage split (W^T parts in shared memory, X's parts in TMEM)
    B_EMPTY = 8,                   // 4: stage's MMAs finished (its shared memory and TMEM slot are free)
    B_ACCF = 12,                   // 2: accumulator holds a finished partial sum
    B_ACCE = 14,                   // 2: accumulator read by the epilogue
    B_STALL = 16,                  // test hook: nothing arrives here (see Params::stall)
    B_COUNT = 17
};

// mode 0: the Q, K, V projection.
// mode 1: dQ = dS K of the causal backward for every (batch, head): A = dS
//   [bh][T rows][T keys] (zero above the diagonal), B = that head's K
//   transposed and split (K^T high / low [bh][d][Tp]), C = dQ in the activation
//   layout; an item is one 128-row tile of one (batch, head) and reads keys
//   0 .. min(m0 + 128, T) only.
// mode 2: dV = P^T dO or dK = dS^T Q: as mode 1 with A = P^T or dS^T [bh][T
//   keys][T queries] (zero left of the diagonal), reading queries m0 .. T only.
// mode 3: the scores X = Q K^T or Y = dO V^T per (batch, head), 128 x 128 tiles
//   at or below the diagonal: A = Q or dO read raw in the activation layout, B =
//   K or V split by rows ([bh][T][d] high / low), C = the tile of a
//   [bh][T][T] buffer.
struct Params {
    const float *bias[3];
    int M, N, K;                   // (N: out_features, K: in_features; modes 1-2: T, d, T; mode 3: T, T, d)
    int mode, H, D;                // modes 1-3: heads (bh = b * H + h), head dim
    int mt, nt;                    // row tiles, column tiles per output
    int n_items, nk;
    int *err;
    int fold;                      // k stages per fresh TMEM sum (a power of two)
    int stall;                     // test hook: the MMA warp first waits on B_STALL for
    long long stall_limit;         // stall_limit SM cycles (the other waits keep their bound)
};

// mode 0: output w, rows m0.., columns n0..; mode 1: w = (batch, head) index,
// n0 = 0, items longest first (the last row tiles read the most keys)
__device__ __forceinline__ void item_coords(const Params &p, int item, int &m0, int &w, int &n0) {
    if (p.mode == 3) {                             // (bh, query tile qt, key tile kt <= qt)
        const int pairs = p.mt * (p.mt + 1) / 2;
        w = item / pairs;
        const int r = item % pairs;
        int qt = (int)((sqrtf(8.f * (float)r + 1.f) - 1.f) * 0.5f);
        while (qt * (qt + 1) / 2 > r) qt--;
        while ((qt + 1) * (qt + 2) / 2 <= r) qt++;
        m0 = qt * BM;
        n0 = (r - qt * (qt + 1) / 2) * BN;
        return;
    }
    if (p.mode == 1 || p.mode == 2) {              // longest first: mode 1's last tiles, mode 2's first
        const int bhn = p.n_items / p.mt;
        m0 = (p.mode == 1 ? p.mt - 1 - item / bhn : item / bhn) * BM;
        w = item % bhn;
        n0 = 0;
        return;
    }
    const int ng = item / p.mt;                    // consecutive CTAs share a column tile of W
    m0 = (item % p.mt) * BM;
    w = ng / p.nt;
    n0 = (ng % p.nt) * BN;
}
// k stages of an item, and its first k stage
__device__ __forceinline__ int item_nk(const Params &p, int m0) {
    if (p.mode == 1) return (min(m0 + BM, p.K) + BK - 1) / BK;
    if (p.mode == 2) return (p.K + BK - 1) / BK - m0 / BK;
    return p.nk;
}
__device__ __forceinline__ int item_k0(const Params &p, int m0) { return p.mode == 2 ? m0 / BK : 0; }

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

// The high part is x rounded to the nearest tf32 value (its 13 low mantissa
// bits cleared after adding half of their weight), so the low part x - xh,
// exact in fp32, is at most half a tf32 step: the MMA's tf32 view of it then
// loses at most 2^-23 of x, where clearing the bits without rounding loses
// up to 2^-21 (and the dropped xl * yl term shrinks from 2^-20 to 2^-22).
__device__ __forceinline__ float hi_part(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// W (K x N, row-major, one of three) -> rows [w*N, (w+1)*N) of W^T high and
// low (3N x Kp).  A block moves a 32 x 32 tile through shared memory: reads
// are coalesced along n, writes along k.
__global__ void __launch_bounds__(256)
qkv_split_w_kernel(const float *__restrict__ w0, const float *__restrict__ w1, const float *__restrict__ w2,
                   float *__restrict__ wth, float *__restrict__ wtl, int K, int N, long long Kp)
{
    pdl_begin();   // launched by launch_pdl
    __shared__ float tile[32][33];
    const int w = blockIdx.z;
    const float *src = w == 0 ? w0 : w == 1 ? w1 : w2;
    const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int k = k0 + ty + 8 * i, n = n0 + tx;
        tile[ty + 8 * i][tx] = (k < K && n < N) ? __ldg(src + (long long)k * N + n) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int n = n0 + ty + 8 * i, k = k0 + tx;
        if (n < N && k < K) {
            const float x = tile[tx][ty + 8 * i], h = hi_part(x);
            const long long o = ((long long)w * N + n) * Kp + k;
            wth[o] = h;
            wtl[o] = x - h;
        }
    }
}

// The operand splits of the backward GEMMs in one launch, over 32 x 32 tiles
// (rows j, head columns n) of every (batch, head) of a tensor in the activation
// layout (row b*T + j, columns h*D .. h*D + D - 1, rows in_stride floats
// apart).  Tensor z is written split by rows, [bh][T][D] high and low (the
// K-major B operands of the score GEMMs), where rh[z] is set, and transposed and
// split, [bh][D][Tp] (the B operands of dQ = dS K, dV = P^T dO, dK = dS^T Q),
// where th[z] is set: K both ways, Q and dO transposed, V by rows.
struct SplitOperands {
    const float *src[4];
    float *rh[4], *rl[4], *th[4], *tl[4];
};
__global__ void __launch_bounds__(256)
split_operands_kernel(const __grid_constant__ SplitOperands a, long long in_stride, int T, int H, int D, long long Tp)
{
    pdl_begin();   // launched by launch_pdl
    __shared__ float tile[32][33];
    const int z = blockIdx.z, bh = blockIdx.y;
    const int ntn = (D + 31) / 32;
    const int n0 = (int)(blockIdx.x % ntn) * 32, j0 = (int)(blockIdx.x / ntn) * 32;
    const float *src = a.src[z] + (long long)(bh / H) * T * in_stride + (long long)(bh % H) * D;
    float *rh = a.rh[z], *rl = a.rl[z], *th = a.th[z], *tl = a.tl[z];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int j = j0 + ty + 8 * i, n = n0 + tx;
        const bool in = j < T && n < D;
        const float x = in ? __ldg(src + (long long)j * in_stride + n) : 0.f;
        tile[ty + 8 * i][tx] = x;
        if (rh != nullptr && in) {
            const float hh = hi_part(x);
            const long long o = ((long long)bh * T + j) * D + n;
            rh[o] = hh;
            rl[o] = x - hh;
        }
    }
    if (th == nullptr) return;                       // (the whole block: z is uniform)
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int n = n0 + ty + 8 * i, j = j0 + tx;
        if (n < D && j < T) {
            const float x = tile[tx][ty + 8 * i], hh = hi_part(x);
            const long long o = ((long long)bh * D + n) * Tp + j;
            th[o] = hh;
            tl[o] = x - hh;
        }
    }
}

// From the score tiles X = Q K^T (buf1) and Y = dO V^T (buf2), both [bh][T][T]
// with rows i and keys j: P = 2^(X log2(e)/sqrt(d) - lse2_i) and
// dS = P (Y - D_i) / sqrt(d), 0 for j > i (train.c:385-400 restated on the
// saved row statistics).  dS (rows i) goes to `ds`; P^T and dS^T (rows j) to
// the mirror tile (kt, qt) of buf1 and buf2 -- above the diagonal, where no
// score tile lives.  A CTA takes the 64-key half h of an off-diagonal tile
// (the halves read and write disjoint regions), or both halves of a diagonal
// tile one after the other: there half 0's mirror writes land on rows 0-63,
// which half 1 only has masked entries in, and half 1's on rows 64-127 after
// half 0 has read them.  Units of a (batch, head): qt^2 + 2 kt + h for the
// halves of tile (qt, kt < qt), qt^2 + 2 qt for the diagonal tile qt.
constexpr int kSgCols = 64;                        // keys per half tile
constexpr int kSgLd = kSgCols + 1;                 // padded shared row (odd: conflict-free columns)
constexpr int kSgThreads = 512;
constexpr int kSgIters = BM * (kSgCols / 4) / kSgThreads;   // float4 of a half tile per thread and operand
static_assert(kSgThreads == 32 * (kSgCols / 4) && kSgIters * 32 == BM, "thread t: rows t/16 + 32 it, keys 4 (t % 16)");
static_assert(kSgThreads / 32 * 4 == kSgCols && BM == 4 * 32, "mirror: warp w columns 4w..4w+3, lane rows l + 32 m");
// Two CTAs per SM at 64 registers: at the trainer shape this ran faster than three CTAs
// at 40 registers with spills, and than rows of 4 x 128 bytes (conflict-free shared stores)
// in place of 2 x 256.
__global__ void __launch_bounds__(kSgThreads, 2)
scores_to_grads_kernel(float *__restrict__ buf1, float *__restrict__ buf2, const float *__restrict__ lse2,
                       const float *__restrict__ dvec, float *__restrict__ ds, int T, int mt, float qk_scale,
                       float ds_scale)
{
    pdl_begin();   // launched by launch_pdl
    extern __shared__ float sg[];
    float *sx = sg, *sy = sg + BM * kSgLd;
    __shared__ float rl[BM], rd[BM];
    const int bh = blockIdx.y;
    const int r = blockIdx.x;
    int qt = (int)sqrtf((float)r);
    while (qt * qt > r) qt--;
    while ((qt + 1) * (qt + 1) <= r) qt++;
    const int rem = r - qt * qt;
    const bool diag = rem == 2 * qt;
    const int kt = diag ? qt : rem >> 1;
    const int i0 = qt * BM;
    const long long base = (long long)bh * T * T;
    if (threadIdx.x < BM) {
        const int i = i0 + threadIdx.x;
        rl[threadIdx.x] = i < T ? lse2[(long long)bh * T + i] : 0.f;
        rd[threadIdx.x] = i < T ? dvec[(long long)bh * T + i] : 0.f;
    }
    for (int hh = diag ? 0 : (rem & 1); hh < (diag ? 2 : (rem & 1) + 1); hh++) {
        const int j0 = kt * BN + hh * kSgCols;
        // 128 rows x 64 keys as 16 float4 per row (T % 4 == 0: a float4 is all in or all out);
        // thread t takes rows t/16 + 32 it, keys 4 (t % 16) .. +3, and issues all its loads of
        // the half before it uses any
        const int a0 = threadIdx.x >> 4, c = (threadIdx.x & 15) * 4, j = j0 + c;
        const long long off0 = base + (long long)(i0 + a0) * T + j;
        float4 xr[kSgIters], yr[kSgIters];
#pragma unroll
        for (int it = 0; it < kSgIters; it++) {
            const int i = i0 + a0 + 32 * it;
            const long long off = off0 + (long long)(32 * it) * T;
            xr[it] = make_float4(0.f, 0.f, 0.f, 0.f);
            yr[it] = xr[it];
            if (i < T && j < T && j <= i + 3) {        // (a float4 wholly above the diagonal is not read)
                xr[it] = *reinterpret_cast<const float4 *>(buf1 + off);
                yr[it] = *reinterpret_cast<const float4 *>(buf2 + off);
            }
        }
        __syncthreads();                               // (row statistics loaded; the previous half's tiles free)
        // P and dS in registers (over the loaded values); dS (rows i) straight to `ds`, both into
        // shared memory for the mirror
#pragma unroll
        for (int it = 0; it < kSgIters; it++) {
            const int a = a0 + 32 * it, i = i0 + a;
            const float la = rl[a], da = rd[a];
            float *px = sx + a * kSgLd + c, *py = sy + a * kSgLd + c;
            auto grad = [&](float &x, float &y, int e) {
                const bool live = i < T && j + e <= i;
                x = live ? exp2f(x * qk_scale - la) : 0.f;
                y = live ? x * (y - da) * ds_scale : 0.f;
                px[e] = x;
                py[e] = y;
            };
            grad(xr[it].x, yr[it].x, 0);
            grad(xr[it].y, yr[it].y, 1);
            grad(xr[it].z, yr[it].z, 2);
            grad(xr[it].w, yr[it].w, 3);
            if (i < T && j < T)
                *reinterpret_cast<float4 *>(ds + off0 + (long long)(32 * it) * T) = yr[it];
        }
        __syncthreads();
        // P^T and dS^T (rows j): warp w writes columns 4w .. 4w+3 of the tiles, lane l rows
        // l + 32 m (conflict-free shared reads, 128-byte rows of the mirror per instruction)
        {
            const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const int cc = 4 * w + (k >> 2), a = l + 32 * (k & 3);
                const int i = i0 + a, jj = j0 + cc;
                if (i < T && jj < T) {
                    const long long o = base + (long long)jj * T + i;
                    buf1[o] = sx[a * kSgLd + cc];
                    buf2[o] = sy[a * kSgLd + cc];
                }
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1)
qkv_tf32_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap twh,
                const __grid_constant__ CUtensorMap twl, const __grid_constant__ CUtensorMap to0,
                const __grid_constant__ CUtensorMap to1, const __grid_constant__ CUtensorMap to2,
                const __grid_constant__ Params p)
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
        mbar_init(BAR(B_STALL), 1);
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
                prefetch_tmap(&twh);
                prefetch_tmap(&twl);
            }
            int g = 0;                                       // stages issued
            bool ok = true;
            for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
                int m0, w, n0;
                item_coords(p, item, m0, w, n0);
                const int wrow = w * p.N + n0;               // rows of W^T (rows past N read the next
                                                             // weight's or zeros; their columns are not stored)
                const int nk = item_nk(p, m0), k0 = item_k0(p, m0);
                for (int ks = 0; ks < nk; ks++, g++) {
                    const int st = g % kStages;
                    if (g >= kStages && !(ok = wait_w(B_EMPTY + st, g / kStages - 1, 0x501))) break;
                    if (leader) {
                        const uint32_t s0 = base + st * STAGE;
                        const int kx = (k0 + ks) * BK;
                        mbar_arrive_expect_tx(BAR(B_FULL + st), XB + 2 * WB);
                        if (p.mode == 1 || p.mode == 2) {    // 3-D maps over the (batch, head) index
                            tma_load_3d(s0 + OFF_X, &tx, BAR(B_FULL + st), kx, m0, w);
                            tma_load_3d(s0 + OFF_WH, &twh, BAR(B_FULL + st), kx, 0, w);
                            tma_load_3d(s0 + OFF_WL, &twl, BAR(B_FULL + st), kx, 0, w);
                        } else if (p.mode == 3) {            // A raw in the activation layout
                            tma_load_3d(s0 + OFF_X, &tx, BAR(B_FULL + st), (w % p.H) * p.D + kx, m0, w / p.H);
                            tma_load_3d(s0 + OFF_WH, &twh, BAR(B_FULL + st), kx, n0, w);
                            tma_load_3d(s0 + OFF_WL, &twl, BAR(B_FULL + st), kx, n0, w);
                        } else {
                            tma_load_2d(s0 + OFF_X, &tx, BAR(B_FULL + st), ks * BK, m0);
                            tma_load_2d(s0 + OFF_WH, &twh, BAR(B_FULL + st), ks * BK, wrow);
                            tma_load_2d(s0 + OFF_WL, &twl, BAR(B_FULL + st), ks * BK, wrow);
                        }
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
            if (p.stall)         // the bounded wait runs out: code 0x5ff, abort flag, every role stops
                ok = __all_sync(0xffffffffu, mbar_wait(BAR(B_STALL), 0u, abort_flag, p.err, 0x5ff, p.stall_limit));
            for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
                int m0, w, n0;
                item_coords(p, item, m0, w, n0);
                const int nk = item_nk(p, m0);
                for (int ks = 0; ks < nk; ks++, g++) {
                    const int a = ch & 1;
                    const int kf = ks & (p.fold - 1);      // stage within the TMEM sum
                    if (kf == 0 && ch >= 2 && !(ok = wait_w(B_ACCE + a, ch / 2 - 1, 0x511))) break;
                    const int st = g % kStages;
                    if (!(ok = wait_w(B_SPLIT + st, g / kStages, 0x512))) break;
                    tc_fence_after();
                    const uint32_t s0 = base + st * STAGE;
                    if (leader) {
#pragma unroll
                        for (int part = 0; part < 3; part++) {       // hh, hl, lh
                            const uint32_t xa = tmem + TM_X + 64 * st + (part == 2 ? 32 : 0);
                            const uint32_t wb = s0 + (part == 1 ? OFF_WL : OFF_WH);
#pragma unroll
                            for (int kk = 0; kk < BK / 8; kk++)
                                mma_tf32_ts(tmem + BN * a, xa + 8 * kk, sw128_desc(wb + 32 * kk, 16, 1024), idD,
                                            (kf > 0 || part > 0 || kk > 0));
                        }
                        mma_commit(BAR(B_EMPTY + st));
                    }
                    const bool last = kf == p.fold - 1 || ks == nk - 1;
                    if (last) {
                        if (leader) mma_commit(BAR(B_ACCF + a));
                        ch++;
                    }
                    __syncwarp();
                }
            }
        } else if (warp >= 4) {
            // -------------------------------------------------------- splitters
            int g = 0;
            bool ok = true;
            for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
                int m0, w, n0;
                item_coords(p, item, m0, w, n0);
                const int nk = item_nk(p, m0);
                for (int ks = 0; ks < nk; ks++, g++) {
                    const int st = g % kStages;
                    if (!(ok = wait_w(B_FULL + st, g / kStages, 0x521))) break;
                    uint8_t *s0 = sb + st * STAGE;
                    tc_fence_after();
                    // X: this warp's 32 rows (its TMEM lane quadrant), one row per thread
                    // (128 bytes, 128-byte swizzle) -> high and low parts in the stage's
                    // TMEM slot.  The slot is free: the stage's previous MMAs finished
                    // before its TMA load was issued.
                    {
                        const int quad = warp & 3, row = quad * 32 + lane;
                        uint32_t hi[32], lo[32];
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const float4 x = *reinterpret_cast<const float4 *>(s0 + OFF_X + row * 128 + ((j ^ (row & 7)) << 4));
                            const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                            for (int u = 0; u < 4; u++) {
                                const float h = hi_part(xv[u]);
                                hi[4 * j + u] = __float_as_uint(h);
                                lo[4 * j + u] = __float_as_uint(xv[u] - h);
                            }
                        }
                        const uint32_t t = tmem + ((uint32_t)(quad * 32) << 16) + TM_X + 64 * st;
                        tmem_st32(t, hi);
                        tmem_st32(t + 32, lo);
                    }
                    tmem_wait_st();
                    tc_fence_before();
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
        float acc[BN];
        int ch = 0;
        bool ok = true;
        for (int item = blockIdx.x; ok && item < p.n_items; item += gridDim.x) {
            int m0, w, n0;
            item_coords(p, item, m0, w, n0);
            const int nchunks = (item_nk(p, m0) + p.fold - 1) / p.fold;
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
            const float *bias = p.mode != 0 ? nullptr : p.bias[w];
            const CUtensorMap *mo = p.mode != 0 || w == 0 ? &to0 : w == 1 ? &to1 : &to2;
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
                    if (p.mode == 1 || p.mode == 2)   // dQ / dK / dV rows b*T + i, columns h*d + n
                        tma_store_3d(mo, smem_u32(buf), (w % p.H) * p.N + col0, m0 + 32 * quad, w / p.H);
                    else if (p.mode == 3)             // the score tile of the [bh][T][T] buffer
                        tma_store_3d(mo, smem_u32(buf), col0, m0 + 32 * quad, w);
                    else
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

// Workspace of the split weights: W^T high then W^T low, each 3N x Kp floats.
static long long qkv_kp(const attn_qkv_shape *s) { return ((long long)s->in_features + 3) / 4 * 4; }
static size_t qkv_ws_half(const attn_qkv_shape *s) {
    return ((size_t)3 * s->out_features * (size_t)qkv_kp(s) * 4 + 255) / 256 * 256;
}
static size_t qkv_ws_bytes(const attn_qkv_shape *s) { return 2 * qkv_ws_half(s); }

// Library-owned workspaces, one per (device, slot), grown on demand; calls that
// use one must not overlap on the GPU.  Slot 0: the QKV projection's split
// weights; slot 1: the drop-in backward's score buffers, splits and row
// statistics; slot 3: fp32 copies for the bf16 forward at d 32/96/128.
void *library_workspace(int which, size_t bytes, cudaStream_t s) {
    static std::mutex mu;
    static std::map<std::pair<int, int>, std::pair<void *, size_t>> pool;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    auto &slot = pool[std::make_pair(dev, which)];
    if (slot.second >= bytes) return slot.first;
    if (slot.first) {
        cudaStreamSynchronize(s);
        cudaFree(slot.first);
        slot = {nullptr, 0};
    }
    void *ptr = nullptr;
    if (cudaMalloc(&ptr, bytes) != cudaSuccess) return nullptr;
    slot = {ptr, bytes};
    return ptr;
}

// Test hook (attn_debug_qkv_timeout): the next `g_qkv_stall` launches stall.
static std::atomic<int> g_qkv_stall{0};
static std::atomic<long long> g_qkv_stall_limit{0};

int launch_qkv_tf32_sm100(const attn_qkv_shape *s, const float *x, const float *const w[3],
                          const float *const bias[3], float *const out[3], void *ws, int *err, cudaStream_t stream) {
    using namespace attn::qkv;
    const long long ldx = s->x_row_stride ? s->x_row_stride : s->in_features;
    const long long ldo = s->out_row_stride ? s->out_row_stride : s->out_features;
    const long long Kp = qkv_kp(s);
    const size_t half = qkv_ws_half(s);
    float *wth = static_cast<float *>(ws);
    float *wtl = reinterpret_cast<float *>(static_cast<char *>(ws) + half);
    CUtensorMap mx, mwh, mwl, mo[3];
    if (!map_2d(&mx, x, s->in_features, s->rows, ldx, BK, BM) ||
        !map_2d(&mwh, wth, s->in_features, 3LL * s->out_features, Kp, BK, BN) ||
        !map_2d(&mwl, wtl, s->in_features, 3LL * s->out_features, Kp, BK, BN))
        return set_error(ATTN_ERR_CUDA, "QKV projection: cuTensorMapEncodeTiled failed (X or W)");
    for (int i = 0; i < 3; i++)
        if (!map_2d(&mo[i], out[i], s->out_features, s->rows, ldo, 32, 32))
            return set_error(ATTN_ERR_CUDA, "QKV projection: cuTensorMapEncodeTiled failed (output)");
    Params p;
    for (int i = 0; i < 3; i++) p.bias[i] = bias[i];
    p.M = s->rows;
    p.N = s->out_features;
    p.K = s->in_features;
    p.mode = 0;
    p.H = 0;
    p.D = 0;
    p.fold = kFoldQKV;
    p.mt = (p.M + BM - 1) / BM;
    p.nt = (p.N + BN - 1) / BN;
    p.n_items = 3 * p.mt * p.nt;
    p.nk = (p.K + BK - 1) / BK;
    p.err = err;
    p.stall = 0;
    p.stall_limit = 0;
    if (g_qkv_stall.load() > 0) {
        g_qkv_stall.fetch_sub(1);
        p.stall = 1;
        p.stall_limit = g_qkv_stall_limit.load();
    }
    const dim3 sgrid((p.N + 31) / 32, (p.K + 31) / 32, 3);
    int st = check_pdl(launch_pdl(qkv_split_w_kernel, sgrid, dim3(256), 0, stream, w[0], w[1], w[2], wth, wtl, p.K,
                                  p.N, Kp),
                       "QKV projection: weight split kernel");
    if (st != ATTN_OK) return st;
    const int ctas = std::max(1, std::min(sm_count_here(), p.n_items));
    if (!ensure_smem_attr((const void *)qkv_tf32_kernel, SMEM))
        return set_error(ATTN_ERR_CUDA, "QKV projection: cannot set shared-memory size");
    if (!ensure_carveout((const void *)qkv_tf32_kernel, 100))
        return set_error(ATTN_ERR_CUDA, "QKV projection: cannot set the shared-memory carveout");
    return check_pdl(launch_pdl(qkv_tf32_kernel, dim3(ctas), dim3(kThreads), (size_t)SMEM, stream, mx, mwh, mwl,
                                mo[0], mo[1], mo[2], p),
                     "QKV projection kernel");
}

// 3-D view {cols, rows, batch} of fp32 data, boxes of box_cols x box_rows x 1
// with the 128-byte swizzle.
static bool map_3d(CUtensorMap *m, const void *ptr, long long cols, long long rows, long long batch,
                   long long row_stride, long long batch_stride, int box_cols, int box_rows) {
    auto fn = encode_fn_qkv();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batch};
    cuuint64_t strides[2] = {(cuuint64_t)row_stride * 4, (cuuint64_t)batch_stride * 4};
    cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------------------
// fp32 backward at d 96 / 128 with every product on the tensor cores
// ---------------------------------------------------------------------------
int launch_bwd_rowdot(int dtype, int D, const void *o, const void *dout, const float *lse, float *ws,
                      long long in_stride, long long out_stride, int B, int H, int T, cudaStream_t s);

namespace {
struct BwdTcLayout {
    size_t off[14];
    size_t total;
    BwdTcLayout(int B, int H, int T, int D) {
        const size_t BH = (size_t)B * H, Tp = ((size_t)T + 3) / 4 * 4;
        const size_t sz[14] = {2 * BH * T,                                   // lse2, D
                               BH * T * D, BH * T * D, BH * T * D, BH * T * D, // K, V rows: high, low
                               BH * D * Tp, BH * D * Tp, BH * D * Tp,          // K^T, Q^T, dO^T high
                               BH * D * Tp, BH * D * Tp, BH * D * Tp,          //              low
                               BH * T * T, BH * T * T, 0};                     // buf1, buf2
        size_t o = 0;
        for (int i = 0; i < 14; i++) {
            off[i] = o;
            o += (sz[i] * 4 + 255) / 256 * 256;
        }
        total = o;
    }
};
}  // namespace

size_t bwd_tc_ws_bytes(int B, int H, int T, int D) { return BwdTcLayout(B, H, T, D).total; }

static int launch_gemm_mode(int mode, const CUtensorMap &a, const CUtensorMap &bh, const CUtensorMap &bl,
                            const CUtensorMap &out, int T, int H, int D, long long BH, int *err, cudaStream_t stream) {
    using namespace attn::qkv;
    Params p;
    for (int i = 0; i < 3; i++) p.bias[i] = nullptr;
    p.mode = mode;
    p.H = H;
    p.D = D;
    p.fold = kFoldBwd;
    p.M = T;
    p.mt = (T + BM - 1) / BM;
    if (mode == 3) {
        p.N = T;
        p.K = D;
        p.nt = p.mt;
        p.n_items = (int)(BH * p.mt * (p.mt + 1) / 2);
        p.nk = (D + BK - 1) / BK;
    } else {
        p.N = D;
        p.K = T;
        p.nt = 1;
        p.n_items = (int)(BH * p.mt);
        p.nk = (T + BK - 1) / BK;
    }
    p.err = err;
    p.stall = 0;
    p.stall_limit = 0;
    const int ctas = std::max(1, std::min(sm_count_here(), p.n_items));
    if (!ensure_smem_attr((const void *)qkv_tf32_kernel, SMEM) || !ensure_carveout((const void *)qkv_tf32_kernel, 100))
        return set_error(ATTN_ERR_CUDA, "tensor-core backward: cannot set the GEMM kernel's shared memory");
    return check_pdl(launch_pdl(qkv_tf32_kernel, dim3(ctas), dim3(kThreads), (size_t)SMEM, stream, a, bh, bl, out, out,
                                out, p),
                     "tensor-core backward GEMM");
}

// dQ, dK, dV (SET) from dO, Q, K, V, O and lse at d 96 / 128 with every product
// on the tensor cores (3xTF32): the scores X = Q K^T and Y = dO V^T as GEMM
// tiles at or below the diagonal, P and dS from them, then dQ = dS K,
// dV = P^T dO and dK = dS^T Q as GEMMs that read only their causal k range.
// `ds` is a [B*H][T][T] fp32 buffer (the reference trainer's scratch); ws holds
// bwd_tc_ws_bytes (256-byte aligned).  Needs T % 4 == 0, the strides % 4 == 0,
// 16-byte aligned tensors and B*H <= 65535.
int launch_bwd_tc(int D, const float *dout, const float *q, const float *k, const float *v, const float *o,
                  const float *lse, float *dq, float *dk, float *dv, float *ds, void *ws, long long in_stride,
                  long long out_stride, int B, int H, int T, int *err, cudaStream_t s) {
    using namespace attn::qkv;
    const BwdTcLayout L(B, H, T, D);
    char *w = static_cast<char *>(ws);
    auto F = [&](int i) { return reinterpret_cast<float *>(w + L.off[i]); };
    float *stats = F(0), *krh = F(1), *krl = F(2), *vrh = F(3), *vrl = F(4);
    float *kth = F(5), *qth = F(6), *oth = F(7), *ktl = F(8), *qtl = F(9), *otl = F(10);
    float *buf1 = F(11), *buf2 = F(12);
    const long long BH = (long long)B * H, Tp = ((long long)T + 3) / 4 * 4;
    const float qk_scale = attn::kLog2e / sqrtf((float)D), ds_scale = 1.0f / sqrtf((float)D);
    int st = launch_bwd_rowdot(ATTN_F32, D, o, dout, lse, stats, in_stride, out_stride, B, H, T, s);
    if (st) return st;
    SplitOperands so = {};
    so.src[0] = k, so.rh[0] = krh, so.rl[0] = krl, so.th[0] = kth, so.tl[0] = ktl;
    so.src[1] = q, so.th[1] = qth, so.tl[1] = qtl;
    so.src[2] = dout, so.th[2] = oth, so.tl[2] = otl;
    so.src[3] = v, so.rh[3] = vrh, so.rl[3] = vrl;
    const dim3 sgrid((unsigned)(((D + 31) / 32) * ((T + 31) / 32)), (unsigned)BH, 4);
    if ((st = check_pdl(launch_pdl(split_operands_kernel, sgrid, dim3(256), 0, s, so, in_stride, T, H, D, Tp),
                        "split the operands")))
        return st;
    CUtensorMap mq, mo_, mkh, mkl, mvh, mvl, mb1, mb2, mds, mkth, mktl, mqth, mqtl, moth, motl, ydq, ydk, ydv;
    bool okm = map_3d(&mq, q, (long long)H * D, T, B, in_stride, (long long)T * in_stride, BK, BM) &&
               map_3d(&mo_, dout, (long long)H * D, T, B, in_stride, (long long)T * in_stride, BK, BM) &&
               map_3d(&mkh, krh, D, T, BH, D, (long long)T * D, BK, BN) &&
               map_3d(&mkl, krl, D, T, BH, D, (long long)T * D, BK, BN) &&
               map_3d(&mvh, vrh, D, T, BH, D, (long long)T * D, BK, BN) &&
               map_3d(&mvl, vrl, D, T, BH, D, (long long)T * D, BK, BN) &&
               map_3d(&mkth, kth, T, D, BH, Tp, (long long)D * Tp, BK, BN) &&
               map_3d(&mktl, ktl, T, D, BH, Tp, (long long)D * Tp, BK, BN) &&
               map_3d(&mqth, qth, T, D, BH, Tp, (long long)D * Tp, BK, BN) &&
               map_3d(&mqtl, qtl, T, D, BH, Tp, (long long)D * Tp, BK, BN) &&
               map_3d(&moth, oth, T, D, BH, Tp, (long long)D * Tp, BK, BN) &&
               map_3d(&motl, otl, T, D, BH, Tp, (long long)D * Tp, BK, BN) &&
               map_3d(&ydq, dq, (long long)H * D, T, B, out_stride, (long long)T * out_stride, 32, 32) &&
               map_3d(&ydk, dk, (long long)H * D, T, B, out_stride, (long long)T * out_stride, 32, 32) &&
               map_3d(&ydv, dv, (long long)H * D, T, B, out_stride, (long long)T * out_stride, 32, 32);
    // the [bh][T][T] buffers: read as GEMM A operands (128-row boxes), written as score tiles (32-row boxes)
    CUtensorMap mb1s, mb2s;
    okm = okm && map_3d(&mb1, buf1, T, T, BH, T, (long long)T * T, BK, BM) &&
          map_3d(&mb2, buf2, T, T, BH, T, (long long)T * T, BK, BM) &&
          map_3d(&mds, ds, T, T, BH, T, (long long)T * T, BK, BM) &&
          map_3d(&mb1s, buf1, T, T, BH, T, (long long)T * T, 32, 32) &&
          map_3d(&mb2s, buf2, T, T, BH, T, (long long)T * T, 32, 32);
    if (!okm) return set_error(ATTN_ERR_CUDA, "tensor-core backward: cuTensorMapEncodeTiled failed");
    if ((st = launch_gemm_mode(3, mq, mkh, mkl, mb1s, T, H, D, BH, err, s)) ||       // X = Q K^T
        (st = launch_gemm_mode(3, mo_, mvh, mvl, mb2s, T, H, D, BH, err, s)))        // Y = dO V^T
        return st;
    const int mt = (T + BM - 1) / BM;
    const size_t sg_smem = (size_t)2 * BM * kSgLd * sizeof(float);     // 65 KB (two CTAs per SM)
    if (!ensure_smem_attr((const void *)scores_to_grads_kernel, sg_smem))
        return set_error(ATTN_ERR_CUDA, "tensor-core backward: cannot set shared-memory size");
    if ((st = check_pdl(launch_pdl(scores_to_grads_kernel, dim3(mt * mt, (unsigned)BH), dim3(kSgThreads), sg_smem,
                                   s, buf1, buf2, (const float *)stats, (const float *)(stats + BH * T), ds, T, mt,
                                   qk_scale, ds_scale), "scores to P and dS")))
        return st;
    if ((st = launch_gemm_mode(1, mds, mkth, mktl, ydq, T, H, D, BH, err, s)) ||      // dQ = dS K
        (st = launch_gemm_mode(2, mb1, moth, motl, ydv, T, H, D, BH, err, s)))        // dV = P^T dO
        return st;
    return launch_gemm_mode(2, mb2, mqth, mqtl, ydk, T, H, D, BH, err, s);            // dK = dS^T Q
}

}  // namespace attn_host

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
namespace attn_host {
int *device_error_ptr();
}

extern "C" {

size_t attn_qkv_workspace_bytes(const attn_qkv_shape *s) {
    if (!s || s->in_features < 1 || s->out_features < 1) return 0;
    return attn_host::qkv_ws_bytes(s);
}

int attn_qkv_proj_ex(const attn_qkv_shape *s, const float *x, const float *wq, const float *wk, const float *wv,
                     const float *bq, const float *bk, const float *bv, float *q, float *k, float *v,
                     void *workspace, size_t workspace_bytes, attn_stream_t stream) {
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
    const size_t need = attn_host::qkv_ws_bytes(s);
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    if (workspace) {
        if (workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
            return set_error(ATTN_ERR_WORKSPACE, "QKV projection: workspace needs %zu bytes (256-byte aligned), "
                             "got %zu", need, workspace_bytes);
    } else if (!(workspace = attn_host::library_workspace(0, need, cs))) {
        return set_error(ATTN_ERR_NOMEM, "QKV projection: cannot allocate the %zu-byte workspace", need);
    }
    const float *w[3] = {wq, wk, wv};
    const float *b[3] = {bq, bk, bv};
    float *o[3] = {q, k, v};
    return attn_host::launch_qkv_tf32_sm100(s, x, w, b, o, workspace, attn_host::device_error_ptr(), cs);
}

int attn_debug_qkv_timeout(int launches, long long limit_cycles) {
    if (launches < 0 || (launches > 0 && limit_cycles < 1000))
        return attn_host::set_error(ATTN_ERR_INVALID, "attn_debug_qkv_timeout: launches %d, limit %lld "
                                    "(the limit must be >= 1000 cycles)", launches, limit_cycles);
    attn_host::g_qkv_stall_limit.store(limit_cycles);
    attn_host::g_qkv_stall.store(launches);
    return ATTN_OK;
}

void attn_qkv_proj(const float *X, const float *Wq, const float *Wk, const float *Wv, const float *bq,
                   const float *bk, const float *bv, float *Q, float *K, float *V, int M, int K_, int N) {
    const attn_qkv_shape s = {M, K_, N, 0, 0};
    const int st = attn_qkv_proj_ex(&s, X, Wq, Wk, Wv, bq, bk, bv, Q, K, V, nullptr, 0, nullptr);
    if (st != ATTN_OK) {
        fprintf(stderr, "CUDA error '%s' at attn_qkv_proj\n", attn_last_error());
        exit(1);
    }
}

}  // extern "C"
