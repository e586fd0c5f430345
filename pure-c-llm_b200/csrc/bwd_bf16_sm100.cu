// bwd_bf16_sm100.cu -- causal attention backward on the Blackwell tensor cores.
//
// Semantics: attention_backward, train.c:373-407, with bf16 Q/K/V/dO/dQ/dK/dV
// and fp32 scores, statistics and accumulators:
//   P = exp(S - lse),  dP = dO V^T,  dS = P (dP - D) / sqrt(d),  D_i = dO_i . O_i
//   dV = P^T dO,  dK = dS^T Q,  dQ = dS K
// P is rebuilt from the forward's lse; the row statistics (lse in base 2, D)
// come from the shared rowdot pre-pass into the workspace.
//
// Two deterministic kernels (no atomics).  A unit is one 128-row tile of one
// (batch, head); each kernel is persistent, one CTA per SM walking its units
// in snake order over the units sorted by descending cost.  The fixed tiles
// of a unit go into one of two buffers, so the next unit's load while the
// current unit runs, and the streamed-tile ring and every barrier phase run
// on across units; the accumulators pass to the next unit once the
// elementwise warps have read them out.  12 warps: warp 0 TMA producer;
// warps 1 and 2 MMA issuers
// (warp 1 the S/dP products, warp 2 the accumulations; warp-converged loops,
// the elected lane issues); warp 3 idle; warps 4-7 and 8-11 two elementwise
// warpgroups, one thread per TMEM lane (= one row of the CTA's tile), the
// first taking columns 0-63 of each streamed tile, the second 64-127.
//   dkdv: key tile kt, loops over query tiles i >= kt.  S^T = K Q_i^T and
//         dP^T = V dO_i^T (both operands in shared memory) into TMEM; the
//         warpgroup writes P^T and dS^T as bf16 pairs into TMEM; then
//         dV += P^T dO_i and dK += dS^T Q_i read them from TMEM (A operand)
//         with dO_i / Q_i from shared memory (MN-major B operand).
//   dq:   query tile qt, loops over key tiles j <= qt.  S = Q K_j^T and
//         dP = dO V_j^T, dS into TMEM, dQ += dS K_j.
// The MMA warp issues the next tile's S/dP as soon as the warpgroup has read
// the current ones, so those products overlap the elementwise work.
// Every mbarrier wait is bounded (device error word + abort flag, as in the
// forward kernel).
#include "common.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <functional>
#include <vector>
#include <cudaTypedefs.h>
#include <type_traits>

namespace attn {
namespace fab {

using namespace sm100;

constexpr int BT = 128;           // rows per tile (TMEM lanes) and columns per tile
constexpr int D = 64;             // head_dim covered by these kernels
constexpr int kStages = 3;
constexpr int kThreads = 384;
#ifndef ATTN_BWD_POLY_PAIRS
#define ATTN_BWD_POLY_PAIRS 3
#endif
constexpr int kPolyPairs = ATTN_BWD_POLY_PAIRS;   // exponential pairs (of 8) computed by exp2_poly2 on the FMA pipe
constexpr int TILE_BYTES = BT * D * 2;        // one 128 x 64 bf16 tile (16 KB)

// TMEM columns (both kernels): X = S or S^T, Y = dP or dP^T (fp32, 128 each),
// A1/A2 accumulators (fp32, 64 each), W1/W2 bf16-pair operands (64 each)
constexpr int TM_X = 0, TM_Y = 128, TM_A1 = 256, TM_A2 = 320, TM_W1 = 384, TM_W2 = 448, TM_COLS = 512;

// barrier slots
//   FIX/FE: fixed tiles of a buffer loaded / free (their unit's last X/Y products done);
//   SF/SE: streamed stage loaded / free; XY: X, Y of a tile ready; XYE: read;
//   W: bf16 operands written; ACC: a tile's accumulations done; ST: statistics
//   staged; AF: the unit's accumulators read out
enum { B_FIX = 0, B_SF = 2, B_SE = 2 + kStages, B_XY = 2 + 2 * kStages, B_XYE, B_W, B_ACC, B_ST, B_FE, B_AF = B_FE + 2,
       B_COUNT };
static_assert(B_COUNT * 8 <= 128, "barrier area");

struct Params {
    void *out1, *out2;           // dkdv: dK, dV;  dq: dQ
    const float *lse2, *dvec;    // [B][H][T]
    long long out_stride;
    int T, H, B, accumulate;
    int n_units;                 // B * H * tiles (see unit_of in the kernel)
    float scale_log2;            // log2(e) / sqrt(d)
    float ds_scale;              // 1 / sqrt(d)
    int *err;
};

struct Smem {
    uint32_t base;
    uint8_t *ptr;
};

template <int N>
__device__ __forceinline__ void store_row_bf16(__nv_bfloat16 *dst, const uint32_t (&acc)[N], bool accumulate) {
#pragma unroll
    for (int c = 0; c < N; c += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = __uint_as_float(acc[c + u]);
        if (accumulate) {
            const uint4 old = *reinterpret_cast<const uint4 *>(dst + c);
            const uint32_t w[4] = {old.x, old.y, old.z, old.w};
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const __nv_bfloat162 pr = *reinterpret_cast<const __nv_bfloat162 *>(&w[u]);
                v[2 * u] += __low2float(pr);
                v[2 * u + 1] += __high2float(pr);
            }
        }
        uint4 o;
        o.x = pack_bf16(v[0], v[1]);
        o.y = pack_bf16(v[2], v[3]);
        o.z = pack_bf16(v[4], v[5]);
        o.w = pack_bf16(v[6], v[7]);
        *reinterpret_cast<uint4 *>(dst + c) = o;
    }
}

// KIND 0: dkdv (fixed tiles K, V; streamed Q_i, dO_i), KIND 1: dq (fixed Q, dO;
// streamed K_j, V_j).  Tensor maps: m_a/m_b are the fixed pair, m_c/m_d the
// streamed pair, all 3-D {H*D, T, B} views with 64 x 128 boxes, 128B swizzle.
template <int KIND>
__global__ void __launch_bounds__(kThreads, 1)
bwd_kernel(const __grid_constant__ CUtensorMap m_a, const __grid_constant__ CUtensorMap m_b,
           const __grid_constant__ CUtensorMap m_c, const __grid_constant__ CUtensorMap m_d, const Params p)
{
    pdl_begin();   // launched by launch_pdl
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *sb = smem_raw + (base - raw);
    // layout: 2 buffers x fixed (A, B), stages x (C, D), row statistics, barriers
    const uint32_t sF = base, sST = base + 4 * TILE_BYTES;
    const int OFF_STATS = 4 * TILE_BYTES + kStages * 2 * TILE_BYTES;     // kStages x 2 x 128 floats
    float *stats = reinterpret_cast<float *>(sb + OFF_STATS);
    const int OFF_BAR = OFF_STATS + kStages * 2 * BT * 4;
    const uint32_t bar0 = base + OFF_BAR;
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sb + OFF_BAR + 128);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sb + OFF_BAR + 132);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_t = (p.T + BT - 1) / BT;
    // Persistent: the CTA walks units k = 0, 1, ... in rounds of gridDim.x,
    // snake order (round k takes position blockIdx.x, or gridDim.x-1-blockIdx.x
    // when k is odd), over units ordered by descending cost.  Unit u: tile rank
    // z = u / (B*H); dkdv: key tile kt = z (small kt has the most query tiles);
    // dq: query tile qt = n_t-1-z (large qt has the most key tiles).  (Grouping
    // the units by (batch, head) pairs, for L2 reuse, cut the DRAM traffic at
    // C5 from 0.56 to 0.40 GB but lost 5-7 % to the rounds' imbalance.)
    struct Unit { int h, b, fixed, first, count; };
    auto unit_of = [&](int k, Unit &un) -> bool {
        const int G = (int)gridDim.x;
        const int u = k * G + ((k & 1) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x);
        if (u >= p.n_units) return false;
        const int hb = p.H * p.B, z = u / hb, r = u - z * hb;
        un.h = r % p.H;
        un.b = r / p.H;
        un.fixed = KIND == 0 ? z : n_t - 1 - z;
        un.first = KIND == 0 ? un.fixed : 0;                  // streamed tile range
        un.count = KIND == 0 ? n_t - un.fixed : un.fixed + 1;
        return true;
    };

    if (threadIdx.x == 0) {
        for (int f = 0; f < 2; f++) { mbar_init(BAR(B_FIX + f), 1); mbar_init(BAR(B_FE + f), 1); }
        for (int s = 0; s < kStages; s++) { mbar_init(BAR(B_SF + s), 1); mbar_init(BAR(B_SE + s), 1); }
        mbar_init(BAR(B_XY), 1);
        mbar_init(BAR(B_XYE), 256);
        mbar_init(BAR(B_W), 256);
        mbar_init(BAR(B_ACC), 1);
        mbar_init(BAR(B_ST), 256);
        mbar_init(BAR(B_AF), 256);
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

    // registers: 384 x 168 at launch; warpgroup 0 (TMA, MMA warps) gives back
    // down to 72 so the two elementwise warpgroups can hold 216 each
    // (128 x 72 + 256 x 216 = 384 x 168); each setmaxnreg inside its branch.
    if (warp < 4) regs_dec<72>();
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tmap(&m_a);
            prefetch_tmap(&m_b);
            prefetch_tmap(&m_c);
            prefetch_tmap(&m_d);
            int g = 0;                               // streamed tiles issued (all units)
            bool ok = true;
            Unit un;
            for (int k = 0; ok && unit_of(k, un); k++) {
                // fixed tiles of unit k go to buffer k & 1, free once unit k-2's
                // last X/Y products completed
                const int fb = k & 1;
                if (k >= 2 && !(ok = mbar_wait(BAR(B_FE + fb), ((k >> 1) + 1) & 1, abort_flag, p.err, 0x302)))
                    break;
                const uint32_t fdst = sF + fb * 2 * TILE_BYTES;
                mbar_arrive_expect_tx(BAR(B_FIX + fb), 2 * TILE_BYTES);
                tma_load_3d(fdst, &m_a, BAR(B_FIX + fb), un.h * D, un.fixed * BT, un.b);
                tma_load_3d(fdst + TILE_BYTES, &m_b, BAR(B_FIX + fb), un.h * D, un.fixed * BT, un.b);
                for (int it = 0; it < un.count; it++, g++) {
                    const int st = g % kStages;
                    if (g >= kStages &&
                        !(ok = mbar_wait(BAR(B_SE + st), ((g / kStages) + 1) & 1, abort_flag, p.err, 0x301)))
                        break;
                    mbar_arrive_expect_tx(BAR(B_SF + st), 2 * TILE_BYTES);
                    const uint32_t dst = sST + st * 2 * TILE_BYTES;
                    tma_load_3d(dst, &m_c, BAR(B_SF + st), un.h * D, (un.first + it) * BT, un.b);
                    tma_load_3d(dst + TILE_BYTES, &m_d, BAR(B_SF + st), un.h * D, (un.first + it) * BT, un.b);
                }
            }
        }
    } else if (warp == 1 || warp == 2) {
        // ------------------------------------------------------------ MMA issuers
        // warp 1: X/Y products of each streamed tile; warp 2: the accumulations.
        const bool leader = elect_one();
        auto wait = [&](int b, int parity, int code) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(BAR(b), parity & 1, abort_flag, p.err, code));
        };
        if (warp == 1) {
            constexpr uint32_t idXY = idesc_bf16(BT, BT, 0, 0);    // both operands K-major (along d)
            // X, Y for streamed tile `it`:  dkdv: X = K Q^T, Y = V dO^T;  dq: X = Q K^T, Y = dO V^T
            int g = 0;
            bool ok = true;
            Unit un;
            for (int k = 0; ok && unit_of(k, un); k++) {
                const int fbuf = k & 1;
                if (!(ok = wait(B_FIX + fbuf, k >> 1, 0x311))) break;
                const uint32_t fsrc = sF + fbuf * 2 * TILE_BYTES;
                const uint64_t fa = sw128_desc(fsrc, 16, 1024), fb = sw128_desc(fsrc + TILE_BYTES, 16, 1024);
                for (int it = 0; it < un.count; it++, g++) {
                    if (!(ok = wait(B_SF + g % kStages, g / kStages, 0x312))) break;
                    if (g > 0 && !(ok = wait(B_XYE, g - 1, 0x314))) break;   // X/Y of the previous tile read
                    tc_fence_after();
                    const uint32_t stg = sST + (g % kStages) * 2 * TILE_BYTES;
                    const uint64_t sc = sw128_desc(stg, 16, 1024), sd = sw128_desc(stg + TILE_BYTES, 16, 1024);
                    if (leader) {
#pragma unroll
                        for (int kk = 0; kk < D / 16; kk++)
                            mma_bf16_ss(tmem + TM_X, fa + 2 * kk, sc + 2 * kk, idXY, kk > 0);
#pragma unroll
                        for (int kk = 0; kk < D / 16; kk++)
                            mma_bf16_ss(tmem + TM_Y, fb + 2 * kk, sd + 2 * kk, idXY, kk > 0);
                        mma_commit(BAR(B_XY));
                        if (it == un.count - 1) mma_commit(BAR(B_FE + fbuf));   // the unit's fixed tiles are free
                    }
                    __syncwarp();
                }
            }
        } else {
            constexpr uint32_t idAcc = idesc_bf16(BT, D, 0, 1);    // A from TMEM, B MN-major
            //   dkdv: A1 (dV) += W1 (P^T) . dO_i,  A2 (dK) += W2 (dS^T) . Q_i
            //   dq:   A1 (dQ) += W2 (dS) . K_j
            // (tile it's X/Y products finished before its W was written, so this
            // warp's commit alone frees the stage)
            int g = 0;
            bool ok = true;
            Unit un;
            for (int k = 0; ok && unit_of(k, un); k++)
            for (int it = 0; it < un.count; it++, g++) {
                // the unit's first accumulation overwrites the accumulators: the
                // previous unit's have been read out
                if (it == 0 && k > 0 && !(ok = wait(B_AF, k - 1, 0x316))) break;
                if (!(ok = wait(B_W, g, 0x315))) break;
                tc_fence_after();
                const uint32_t stg = sST + (g % kStages) * 2 * TILE_BYTES;
                if (leader) {
                    if (KIND == 0) {
                        const uint64_t dq_ = sw128_desc(stg, 16384, 1024);                 // Q_i, MN-major
                        const uint64_t ddo = sw128_desc(stg + TILE_BYTES, 16384, 1024);    // dO_i, MN-major
#pragma unroll
                        for (int kk = 0; kk < BT / 16; kk++)
                            mma_bf16_ts(tmem + TM_A1, tmem + TM_W1 + kk * 8, ddo + 128 * kk, idAcc, it > 0 || kk > 0);
#pragma unroll
                        for (int kk = 0; kk < BT / 16; kk++)
                            mma_bf16_ts(tmem + TM_A2, tmem + TM_W2 + kk * 8, dq_ + 128 * kk, idAcc, it > 0 || kk > 0);
                    } else {
                        const uint64_t dk = sw128_desc(stg, 16384, 1024);                  // K_j, MN-major
#pragma unroll
                        for (int kk = 0; kk < BT / 16; kk++)
                            mma_bf16_ts(tmem + TM_A1, tmem + TM_W2 + kk * 8, dk + 128 * kk, idAcc, it > 0 || kk > 0);
                    }
                    mma_commit(BAR(B_ACC));
                    mma_commit(BAR(B_SE + g % kStages));      // streamed stage free
                }
                __syncwarp();
            }
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ elementwise
        regs_inc<216>();
        const int half = (warp - 4) >> 2;            // columns [64 half, 64 half + 64) of each tile
        const int quad = warp & 3;
        const int row = quad * 32 + lane;            // TMEM lane = row of the CTA's fixed tile
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        const uint64_t scale2 = f2(p.scale_log2, p.scale_log2), ds2 = f2(p.ds_scale, p.ds_scale);
        bool ok = true;
        int g = 0;                                   // streamed tiles (all units)
        Unit un;
        for (int k = 0; ok && unit_of(k, un); k++) {
            const int h = un.h, b = un.b, fixed = un.fixed, first = un.first, count = un.count;
            const long long bh = ((long long)b * p.H + h) * p.T;
            const int grow_ = fixed * BT + row;          // global row index of this thread
            float my_nl2 = 0.f, my_ndd = 0.f;            // dq: this query row's -lse2 and -D / sqrt(d)
            if (KIND == 1 && grow_ < p.T) {
                my_nl2 = -__ldg(p.lse2 + bh + grow_);
                my_ndd = -__ldg(p.dvec + bh + grow_) * p.ds_scale;
            }
            for (int it = 0; it < count; it++, g++) {
                const int tcol = first + it;             // streamed tile index
                float *st_l = stats + (g % kStages) * 2 * BT;   // dkdv: lse2 / D of the query columns
                if (KIND == 0) {
                    if (half == 0) {                     // staged as -lse2 and -D / sqrt(d)
                        const int q = tcol * BT + row;
                        st_l[row] = q < p.T ? -__ldg(p.lse2 + bh + q) : 0.f;
                        st_l[BT + row] = q < p.T ? -__ldg(p.dvec + bh + q) * p.ds_scale : 0.f;
                    }
                    // the statistics are in shared memory before anyone reads them (an
                    // mbarrier with a bounded wait, so a warp that gave up on an earlier
                    // wait cannot leave the others blocked here)
                    mbar_arrive(BAR(B_ST));
                    if (!__all_sync(0xffffffffu, mbar_wait(BAR(B_ST), g & 1, abort_flag, p.err, 0x323))) {
                        ok = false;
                        break;
                    }
                }
                ok = mbar_wait(BAR(B_XY), g & 1, abort_flag, p.err, 0x321);
                if (g > 0 && ok) ok = mbar_wait(BAR(B_ACC), (g - 1) & 1, abort_flag, p.err, 0x322);
                if (!(ok = __all_sync(0xffffffffu, ok))) break;
                tc_fence_after();
                const bool diag = (tcol == fixed);
                // this half's 64 columns of X and Y in one round trip
                uint32_t xs[64], ys[64];
    #pragma unroll
                for (int q2 = 0; q2 < 2; q2++) {
                    uint32_t t0[32], t1[32];
                    tmem_ld32(tmem + lb + TM_X + 64 * half + 32 * q2, t0);
                    tmem_ld32(tmem + lb + TM_Y + 64 * half + 32 * q2, t1);
    #pragma unroll
                    for (int c = 0; c < 32; c++) {
                        xs[32 * q2 + c] = t0[c];
                        ys[32 * q2 + c] = t1[c];
                    }
                }
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(BAR(B_XYE));                 // X and Y read: the next products may start
                // P = 2^(S scale - lse2), dS = P (dP - D) / sqrt(d), pairwise on f32x2;
                // the mask (diagonal tile, or key/query columns past T) only where needed
                const bool need_mask = diag || (KIND == 0 && tcol * BT + BT > p.T);
                auto tile = [&](auto masked_tag) {
                    constexpr bool MASKED = decltype(masked_tag)::value;
    #pragma unroll
                    for (int q2 = 0; q2 < 2; q2++) {
                        uint32_t wp[16], wd[16];
    #pragma unroll
                        for (int c = 0; c < 32; c += 2) {
                            const int cc = 32 * q2 + c;      // column within this half
                            const int col = 64 * half + cc;
                            uint64_t nl2, ndd;
                            if (KIND == 0) {                 // row = key, col = query
                                nl2 = *reinterpret_cast<const uint64_t *>(st_l + col);
                                ndd = *reinterpret_cast<const uint64_t *>(st_l + BT + col);
                            } else {                         // row = query, col = key
                                nl2 = f2(my_nl2, my_nl2);
                                ndd = f2(my_ndd, my_ndd);
                            }
                            const uint64_t xa2 = fma2(f2(__uint_as_float(xs[cc]), __uint_as_float(xs[cc + 1])), scale2, nl2);
                            // kPolyPairs of every 8 pairs on the FMA pipe, the rest on MUFU
                            float pv[2];
                            if (((cc >> 1) & 7) < kPolyPairs) {
                                f2_split(exp2_poly2(xa2), pv[0], pv[1]);
                            } else {
                                float a0, a1;
                                f2_split(xa2, a0, a1);
                                pv[0] = ex2(a0);
                                pv[1] = ex2(a1);
                            }
                            if (MASKED) {
    #pragma unroll
                                for (int u = 0; u < 2; u++) {
                                    const int cu = col + u;
                                    const bool m = KIND == 0 ? ((diag && cu < row) || (tcol * BT + cu >= p.T))
                                                             : (diag && cu > row);
                                    if (m) pv[u] = 0.f;
                                }
                            }
                            const uint64_t pv2 = f2(pv[0], pv[1]);
                            const uint64_t t2 = fma2(f2(__uint_as_float(ys[cc]), __uint_as_float(ys[cc + 1])), ds2, ndd);
                            float d0, d1;
                            f2_split(fma2(pv2, t2, 0ull), d0, d1);
                            wp[c / 2] = pack_bf16(pv[0], pv[1]);
                            wd[c / 2] = pack_bf16(d0, d1);
                        }
                        if (KIND == 0) tmem_st16(tmem + lb + TM_W1 + 32 * half + 16 * q2, wp);
                        tmem_st16(tmem + lb + TM_W2 + 32 * half + 16 * q2, wd);
                    }
                };
                if (need_mask) tile(std::true_type{});
                else tile(std::false_type{});
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(BAR(B_W));
            }
            if (!ok) break;
            // epilogue: this half's 32 columns of each accumulator -> global; the
            // accumulators are released to the next unit as soon as they are read
            ok = mbar_wait(BAR(B_ACC), (g - 1) & 1, abort_flag, p.err, 0x324);
            if (!(ok = __all_sync(0xffffffffu, ok))) break;
            tc_fence_after();
            uint32_t acc[2][32];
            tmem_ld32(tmem + lb + TM_A1 + 32 * half, acc[0]);
            if (KIND == 0) tmem_ld32(tmem + lb + TM_A2 + 32 * half, acc[1]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(BAR(B_AF));
            if (grow_ < p.T) {
                for (int a = 0; a < (KIND == 0 ? 2 : 1); a++) {
                    // dkdv: a=0 -> dV (out2), a=1 -> dK (out1);  dq: dQ (out1)
                    void *outp = KIND == 0 ? (a == 0 ? p.out2 : p.out1) : p.out1;
                    __nv_bfloat16 *dst = static_cast<__nv_bfloat16 *>(outp) +
                                         ((long long)b * p.T + grow_) * p.out_stride + (long long)h * D + 32 * half;
                    store_row_bf16<32>(dst, acc[a], p.accumulate != 0);
                }
            }
        }
    }

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

constexpr int smem_bytes() {
    return 4 * TILE_BYTES + kStages * 2 * TILE_BYTES + kStages * 2 * BT * 4 + 256 + 1024;
}

}  // namespace fab
}  // namespace attn

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace attn_host {

bool ensure_smem_attr(const void *func, size_t bytes);
const unsigned short *schedule_get(int kernel_tag, long long key,
                                   const std::function<void(std::vector<unsigned short> &)> &build);
int sm_count_here();
bool ensure_carveout(const void *func, int percent);
int launch_bwd_rowdot(int dtype, int D, const void *o, const void *dout, const float *lse, float *ws,
                      long long in_stride, long long out_stride, int B, int H, int T, cudaStream_t s);

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn_b() {
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

static bool make_map_b(CUtensorMap *m, const void *ptr, int cols, int T, int B, long long stride) {
    struct Entry { const void *ptr; int cols, T, B; long long stride; CUtensorMap map; };
    static thread_local Entry cache[16];
    static thread_local int next = 0;
    for (auto &e : cache)
        if (e.ptr == ptr && e.cols == cols && e.T == T && e.B == B && e.stride == stride) {
            *m = e.map;
            return true;
        }
    auto fn = encode_fn_b();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)stride * 2, (cuuint64_t)stride * 2 * T};
    cuuint32_t box[3] = {64, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    if (fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    cache[next] = Entry{ptr, cols, T, B, stride, *m};
    next = (next + 1) % 16;
    return true;
}

bool bwd_bf16_sm100_supported(int D, long long in_stride, long long out_stride) {
    return D == 64 && in_stride % 8 == 0 && out_stride % 8 == 0 && encode_fn_b() != nullptr;
}

int launch_bwd_bf16_sm100(int D, const void *dout, const void *q, const void *k, const void *v, const void *o,
                          const float *lse, void *dq, void *dk, void *dv, int accumulate, void *ws,
                          long long in_stride, long long out_stride, int B, int H, int T, int *err,
                          cudaStream_t s) {
    using namespace attn::fab;
    if (D != 64) return set_error(ATTN_ERR_UNSUPPORTED, "tcgen05 backward: head_dim %d", D);
    if (((uintptr_t)dout | (uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15)
        return set_error(ATTN_ERR_INVALID, "tcgen05 backward: tensors must be 16-byte aligned");
    int st = launch_bwd_rowdot(ATTN_BF16, D, o, dout, lse, static_cast<float *>(ws), in_stride, out_stride, B, H,
                               T, s);
    if (st) return st;
    CUtensorMap mq, mk, mv, mdo;
    if (!make_map_b(&mq, q, H * D, T, B, in_stride) || !make_map_b(&mk, k, H * D, T, B, in_stride) ||
        !make_map_b(&mv, v, H * D, T, B, in_stride) || !make_map_b(&mdo, dout, H * D, T, B, in_stride))
        return set_error(ATTN_ERR_CUDA, "tcgen05 backward: cuTensorMapEncodeTiled failed");
    Params p;
    p.lse2 = static_cast<const float *>(ws);
    p.dvec = p.lse2 + (long long)B * H * T;
    p.out_stride = out_stride;
    p.T = T;
    p.H = H;
    p.B = B;
    p.accumulate = accumulate;
    p.scale_log2 = attn::kLog2e / sqrtf((float)D);
    p.ds_scale = 1.0f / sqrtf((float)D);
    p.err = err;
    const size_t smem = smem_bytes();
    if (!ensure_smem_attr((const void *)bwd_kernel<0>, smem) || !ensure_smem_attr((const void *)bwd_kernel<1>, smem))
        return set_error(ATTN_ERR_CUDA, "tcgen05 backward: cannot set shared-memory size");
    const int n_t = (T + BT - 1) / BT;
    const long long n_units = (long long)B * H * n_t;
    if (n_units > (1LL << 30)) return set_error(ATTN_ERR_INVALID, "tcgen05 backward: too many tiles");
    p.n_units = (int)n_units;
    const int grid = (int)std::min<long long>(sm_count_here(), n_units);   // persistent
    p.out1 = dk;
    p.out2 = dv;
    // fixed K, V; streamed Q, dO
    if ((st = check_pdl(launch_pdl(bwd_kernel<0>, dim3(grid), dim3(kThreads), smem, s, mk, mv, mq, mdo, p),
                        "tcgen05 backward dkdv kernel")))
        return st;
    p.out1 = dq;
    p.out2 = nullptr;
    // fixed Q, dO; streamed K, V
    return check_pdl(launch_pdl(bwd_kernel<1>, dim3(grid), dim3(kThreads), smem, s, mq, mdo, mk, mv, p),
                     "tcgen05 backward dq kernel");
}

}  // namespace attn_host
