// bwd_tf32_sm100.cu -- causal attention backward for fp32 tensors on the
// Blackwell tensor cores with 3xTF32 products (sm_100a).
//
// Semantics: attention_backward, train.c:373-407, fp32 in and out:
//   P = exp(S - lse),  dP = dO V^T,  dS = P (dP - D) / sqrt(d),  D_i = dO_i . O_i
//   dV = P^T dO,  dK = dS^T Q,  dQ = dS K
// Every product of fp32 values x * y is formed as xh*yh + xh*yl + xl*yh (xh =
// x with its 13 low mantissa bits cleared, exact in tf32; xl = x - xh), so
// results track the fp32 reference to ~1e-6.  P is rebuilt from the forward's
// lse; the row statistics (lse in base 2, D) come from the rowdot pre-pass.
//
// Two deterministic kernels (no atomics), one CTA per 128-row fixed tile of
// one (batch, head), streaming 32-row tiles of the other operand pair:
//   dkdv: fixed K, V; streamed Q_i, dO_i (i from the diagonal to T).
//         X = K Q_i^T, Y = V dO_i^T;  dV += P^T dO_i,  dK += dS^T Q_i
//   dq:   fixed Q, dO; streamed K_j, V_j (j up to the diagonal).
//         X = Q K_j^T, Y = dO V_j^T;  dQ += dS K_j
// The fixed pair's high parts live in TMEM and its low parts in shared memory
// (split in place in the tiles it was loaded into); the X/Y products read
// their A operand from there.  Each streamed tile lands raw in shared memory,
// where splitter warps clear the low bits in place, write the low parts and
// the transposed high and low parts the accumulation products need (all B
// operands K-major).  The elementwise warpgroup writes P and dS high parts
// over X and Y in TMEM and their low parts beside them; the accumulation
// products read them as their A operand.  X/Y and those parts have two TMEM
// buffers (by streamed-tile parity), so the next tile's X/Y products run
// while the elementwise warpgroup works on this one and the tensor core
// accumulates the one before.
// Warps: 0 TMA producer; 1 X/Y issuer; 2 accumulation issuer; 3 idle; 4-7
// splitters; 8-11 elementwise (one thread per TMEM lane = fixed-tile row).
// Every mbarrier wait is bounded (device error word + abort flag).
#include "common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>
#include <type_traits>

namespace attn {
namespace fbt {

using namespace sm100;

constexpr int BT = 128;           // fixed rows per tile (TMEM lanes)
constexpr int BS = 32;            // streamed rows per tile
constexpr int kThreads = 384;
constexpr int kGroupBH = 16;      // (batch, head) pairs per group of the unit order
// The tensor core's accumulation into TMEM is not round-to-nearest; over the
// thousands of products a dK/dV/dQ row gathers at T = 4096 that drifts by
// ~5e-5.  So the accumulators restart every kGroup streamed tiles (96
// accumulation steps, ~4e-6 at worst) and the elementwise warpgroup adds each
// group's sums into fp32 running sums in registers (a thread owns one row).
constexpr int kGroup = 8;

template <int D>
struct Cfg {
    static constexpr int CH = D / 32;               // 128-byte column chunks of a row
    static constexpr int FB = BT * D * 4;           // one raw fixed tile
    static constexpr int SB = BS * D * 4;           // one part of a streamed tile
    // shared memory: the two fixed tiles (raw, then their low parts), 2 stages x
    // (C hi, C lo, C^T hi, C^T lo, D hi, D lo, D^T hi, D^T lo), 2 stages x row
    // statistics (dkdv), barriers
    static constexpr int OFF_FA = 0, OFF_FB = FB;
    static constexpr int OFF_ST = (2 * FB + 1023) / 1024 * 1024;
    static constexpr int STAGE = 8 * SB;
    static constexpr int OFF_STATS = OFF_ST + 2 * STAGE;
    static constexpr int OFF_BAR = OFF_STATS + 2 * 2 * BS * 4;
    static constexpr int SMEM = OFF_BAR + 256 + 1024;
    // TMEM columns: the fixed A and B high parts; two buffers of X, Y (P / dS
    // high parts written over them) and the P and dS low parts; accumulators
    static constexpr int TM_AH = 0, TM_BH = D, TM_XY = 2 * D, XYB = 4 * BS;
    static constexpr int TM_A1 = TM_XY + 2 * XYB, TM_A2 = TM_A1 + D, TM_COLS = 512;
    static_assert(TM_A2 + D <= TM_COLS, "TMEM budget");
    static_assert(SMEM <= 232448, "shared memory");
};
// column of X (0), Y (1), P low (2) or dS low (3) in X/Y buffer b
template <int D>
__device__ __forceinline__ uint32_t xy_col(int b, int which) {
    return (uint32_t)(Cfg<D>::TM_XY + b * Cfg<D>::XYB + which * BS);
}

// barrier slots
enum {
    B_FXF = 0, B_FX, B_SF, B_SS = B_SF + 2, B_SE = B_SS + 2,   // fixed tiles; stages (2 each)
    B_XY = B_SE + 2, B_W = B_XY + 2, B_ACC = B_W + 2,           // per X/Y buffer (2 each)
    B_ST = B_ACC + 2, B_AF, B_COUNT
};

struct Params {
    float *out1, *out2;          // dkdv: dK, dV;  dq: dQ
    const float *lse2, *dvec;    // [B][H][T]
    long long out_stride;
    int T, H, B, accumulate;
    float scale_log2;            // log2(e) / sqrt(d)
    float ds_scale;              // 1 / sqrt(d)
    int *err;
};

__device__ __forceinline__ uint32_t hi_bits(float x) { return __float_as_uint(x) & 0xFFFFE000u; }
__device__ __forceinline__ float f4_at(const float4 &v, int c) {
    return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
}

// KIND 0: dkdv, KIND 1: dq.  m_a/m_b: the fixed pair (128-row boxes), m_c/m_d:
// the streamed pair (32-row boxes); 3-D {H*D, T, B} views, 32-float x rows
// boxes, 128-byte swizzle.
template <int D, int KIND>
__global__ void __launch_bounds__(kThreads, 1)
bwd_tf32_kernel(const __grid_constant__ CUtensorMap m_a, const __grid_constant__ CUtensorMap m_b,
                const __grid_constant__ CUtensorMap m_c, const __grid_constant__ CUtensorMap m_d, const Params p)
{
    pdl_begin();   // launched by launch_pdl
    using C = Cfg<D>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *sb = smem_raw + (base - raw);
    float *stats = reinterpret_cast<float *>(sb + C::OFF_STATS);
    const uint32_t bar0 = base + C::OFF_BAR;
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sb + C::OFF_BAR + 192);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sb + C::OFF_BAR + 196);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_ft = (p.T + BT - 1) / BT;
    // Block u of the 1-D grid: the units come in groups of kGroupBH (batch,
    // head) pairs -- CTAs launched together share a few pairs, whose streamed
    // tiles are read from DRAM about once and then from L2 -- and within a
    // group by descending cost (tile rank z), which keeps each wave's CTAs of
    // similar length.
    const int u = (int)blockIdx.x, hb_all = p.H * p.B;
    const int blk = u / (kGroupBH * n_ft), u_in = u - blk * kGroupBH * n_ft;
    const int hb = min(kGroupBH, hb_all - blk * kGroupBH);
    const int z = u_in / hb, r = blk * kGroupBH + (u_in - z * hb);
    const int h = r % p.H, b = r / p.H;
    // dkdv: key tile kt = z (small kt streams the most query tiles: issued first);
    // dq: query tile qt = n_ft-1-z (large qt streams the most key tiles)
    const int fixed = KIND == 0 ? z : n_ft - 1 - z;
    const int first = KIND == 0 ? fixed * (BT / BS) : 0;                 // streamed tile range
    const int last = KIND == 0 ? (p.T + BS - 1) / BS : (min(p.T, (fixed + 1) * BT) + BS - 1) / BS;
    const int count = last - first;

    if (threadIdx.x == 0) {
        mbar_init(BAR(B_FXF), 1);
        mbar_init(BAR(B_FX), 128);
        for (int s = 0; s < 2; s++) {
            mbar_init(BAR(B_SF + s), 1);
            mbar_init(BAR(B_SS + s), 128);
            mbar_init(BAR(B_SE + s), 1);
        }
        for (int x = 0; x < 2; x++) {
            mbar_init(BAR(B_XY + x), 1);
            mbar_init(BAR(B_W + x), 128);
            mbar_init(BAR(B_ACC + x), 1);
        }
        mbar_init(BAR(B_ST), 128);
        mbar_init(BAR(B_AF), 128);
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
    auto wait_w = [&](int bi, int parity, int code) -> bool {     // warp-wide bounded wait
        return __all_sync(0xffffffffu, mbar_wait(BAR(bi), parity & 1, abort_flag, p.err, code));
    };

    // registers: 384 x 168 at launch; warpgroup 0 gives back down to 64, the
    // splitters down to 144, and the elementwise warpgroup (which keeps its
    // rows' running sums in registers) rises to 256
    // (128 x (64 + 144 + 256) = 59392 <= 384 x 168 = 64512)
    if (warp < 4) regs_dec<64>();
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tmap(&m_a);
            prefetch_tmap(&m_b);
            prefetch_tmap(&m_c);
            prefetch_tmap(&m_d);
            mbar_arrive_expect_tx(BAR(B_FXF), 2 * C::FB);
#pragma unroll
            for (int c = 0; c < C::CH; c++) {
                tma_load_3d(base + C::OFF_FA + c * (BT * 128), &m_a, BAR(B_FXF), h * D + 32 * c, fixed * BT, b);
                tma_load_3d(base + C::OFF_FB + c * (BT * 128), &m_b, BAR(B_FXF), h * D + 32 * c, fixed * BT, b);
            }
            for (int it = 0; it < count; it++) {
                const int st = it & 1;
                if (it >= 2 && !mbar_wait(BAR(B_SE + st), ((it >> 1) + 1) & 1, abort_flag, p.err, 0x501)) break;
                const uint32_t sbase = base + C::OFF_ST + st * C::STAGE;
                const int row = (first + it) * BS;
                mbar_arrive_expect_tx(BAR(B_SF + st), 2 * C::SB);
#pragma unroll
                for (int c = 0; c < C::CH; c++) {
                    tma_load_3d(sbase + c * (BS * 128), &m_c, BAR(B_SF + st), h * D + 32 * c, row, b);            // C hi
                    tma_load_3d(sbase + 4 * C::SB + c * (BS * 128), &m_d, BAR(B_SF + st), h * D + 32 * c, row, b);   // D hi
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ X/Y issuer
        // X = A C^T, Y = B D^T (M = 128 fixed rows, N = 32, K = d) into X/Y buffer
        // it & 1: the high parts of A and B from TMEM, their low parts and C and D
        // (K-major) from shared memory.  The buffer's previous tile (it - 2) must
        // have been accumulated: its P/dS parts live in these columns.
        const bool leader = elect_one();
        constexpr uint32_t idXY = idesc_tf32(BT, BS, 0, 0);
        bool ok = wait_w(B_FX, 0, 0x511);
        for (int it = 0; ok && it < count; it++) {
            const int st = it & 1, xb = it & 1;
            if (!(ok = wait_w(B_SS + st, it >> 1, 0x512))) break;
            if (it >= 2 && !(ok = wait_w(B_ACC + xb, (it >> 1) - 1, 0x513))) break;
            tc_fence_after();
            const uint32_t sbase = base + C::OFF_ST + st * C::STAGE;
            if (leader) {
#pragma unroll
                for (int xy = 0; xy < 2; xy++) {
                    const uint32_t hi = sbase + (xy ? 4 : 0) * C::SB, lo = hi + C::SB;
                    const uint32_t fa_h = tmem + (xy ? C::TM_BH : C::TM_AH);
                    const uint32_t fa_l = base + (xy ? C::OFF_FB : C::OFF_FA);
                    const uint32_t d_t = tmem + xy_col<D>(xb, xy);
#pragma unroll
                    for (int part = 0; part < 3; part++) {       // hh, hl, lh
                        const uint32_t sv = part == 1 ? lo : hi;
#pragma unroll
                        for (int kk = 0; kk < D / 8; kk++) {
                            const uint64_t bd = sw128_desc(sv + (kk >> 2) * (BS * 128) + (kk & 3) * 32, 16, 1024);
                            if (part < 2) {
                                mma_tf32_ts(d_t, fa_h + 8 * kk, bd, idXY, (part > 0 || kk > 0));
                            } else {
                                const uint64_t ad = sw128_desc(fa_l + (kk >> 2) * (BT * 128) + (kk & 3) * 32, 16, 1024);
                                mma_tf32_ss(d_t, ad, bd, idXY, true);
                            }
                        }
                    }
                }
                mma_commit(BAR(B_XY + xb));
            }
            __syncwarp();
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ accumulation issuer
        //   dkdv: A1 (dV) += P^T dO_i,  A2 (dK) += dS^T Q_i;   dq: A1 (dQ) += dS K_j
        // A (P or dS, high over X/Y, low beside) from TMEM; B the transposed
        // streamed tile, K-major: [D rows][32 streamed rows].
        const bool leader = elect_one();
        constexpr uint32_t idAcc = idesc_tf32(BT, D, 0, 0);
        for (int it = 0; it < count; it++) {
            const int st = it & 1, xb = it & 1;
            if (!wait_w(B_W + xb, it >> 1, 0x515)) break;
            // a new group overwrites the accumulators: the previous group's sums were read
            if (it >= kGroup && it % kGroup == 0 && !wait_w(B_AF, it / kGroup - 1, 0x516)) break;
            tc_fence_after();
            const uint32_t sbase = base + C::OFF_ST + st * C::STAGE;
            if (leader) {
#pragma unroll
                for (int a = 0; a < (KIND == 0 ? 2 : 1); a++) {
                    // dkdv a=0: dV from P (X cols) and dO^T;  a=1: dK from dS (Y cols) and Q^T
                    // dq: dQ from dS (Y cols) and K^T
                    const bool use_p = KIND == 0 && a == 0;
                    const uint32_t wh = tmem + xy_col<D>(xb, use_p ? 0 : 1);
                    const uint32_t wl = tmem + xy_col<D>(xb, use_p ? 2 : 3);
                    const uint32_t th = sbase + (use_p ? 6 : 2) * C::SB, tl = th + C::SB;   // (D or C)^T hi, lo
                    const uint32_t acc = tmem + (a ? C::TM_A2 : C::TM_A1);
#pragma unroll
                    for (int part = 0; part < 3; part++) {
                        const uint32_t wa = part == 2 ? wl : wh;
                        const uint32_t tv = part == 1 ? tl : th;
#pragma unroll
                        for (int kk = 0; kk < BS / 8; kk++) {
                            const uint64_t bd = sw128_desc(tv + (kk & 3) * 32, 16, 1024);
                            mma_tf32_ts(acc, wa + 8 * kk, bd, idAcc, (it % kGroup > 0 || part > 0 || kk > 0));
                        }
                    }
                }
                mma_commit(BAR(B_ACC + xb));
                mma_commit(BAR(B_SE + st));             // the stage's X/Y products finished before W
            }
            __syncwarp();
        }
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------------------ splitters
        regs_dec<144>();
        const int quad = warp & 3, row = quad * 32 + lane;
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        bool ok = wait_w(B_FXF, 0, 0x531);
        if (ok) {
            // fixed tiles: high parts -> TMEM, low parts written over the raw values
            // in shared memory (each thread its own row), 16 columns at a time
#pragma unroll 1
            for (int g = 0; g < 2 * 2 * C::CH; g++) {
                const int f = g / (2 * C::CH), c = (g / 2) % C::CH, hh = g & 1;   // tile, chunk, half chunk
                uint32_t hi[16];
                uint8_t *src = sb + (f ? C::OFF_FB : C::OFF_FA) + c * (BT * 128) + row * 128;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    float4 *px = reinterpret_cast<float4 *>(src + (((4 * hh + j) ^ (row & 7)) << 4));
                    const float4 x = *px;
                    const float xv[4] = {x.x, x.y, x.z, x.w};
                    float lv[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const uint32_t hb = hi_bits(xv[u]);
                        hi[4 * j + u] = hb;
                        lv[u] = xv[u] - __uint_as_float(hb);
                    }
                    *px = make_float4(lv[0], lv[1], lv[2], lv[3]);
                }
                tmem_st16(tmem + lb + (f ? C::TM_BH : C::TM_AH) + 32 * c + 16 * hh, hi);
            }
            tmem_wait_st();
            fence_async_smem();                      // the low parts are MMA operands
            tc_fence_before();
            mbar_arrive(BAR(B_FX));
        }
        // streamed tiles: per part (C, D), high in place, low beside it, and the
        // transposed high and low parts (the transpose of D is needed by dkdv
        // only).  Raw tile layout (TMA): chunk c of 32 columns at c*(BS*128),
        // row r at r*128, 16-byte unit u at (u ^ (r & 7)) << 4.  Transposed:
        // [D rows][32 streamed rows], row = column index, same swizzle.
        // By 4x4 micro-blocks with 16-byte loads and stores: a part's 32-row x
        // 32-column block holds an 8x8 grid of them (row group a, column group
        // b), and the 8 lanes of each quarter-warp take one diagonal, b = a + p
        // (mod 8), so their loads and in-place stores hit 8 different 16-byte
        // bank groups of the swizzled rows, and so do their transposed stores.
        constexpr int NMB = 2 * (D / 32) * 64;       // micro-blocks of both parts
        const int tid = threadIdx.x - 128;
        for (int it = 0; ok && it < count; it++) {
            const int st = it & 1;
            if (!(ok = wait_w(B_SF + st, it >> 1, 0x532))) break;
            uint8_t *s0 = sb + C::OFF_ST + st * C::STAGE;
#pragma unroll
            for (int u = 0; u < NMB / 128; u++) {
                const int m = tid + 128 * u, part = m / (NMB / 2), e = m % (NMB / 2);
                const int blk = e >> 6, a = e & 7, bcol = (a + ((e & 63) >> 3)) & 7;
                uint8_t *hi = s0 + (part ? 4 : 0) * C::SB, *lo = hi + C::SB;
                uint8_t *th = hi + 2 * C::SB, *tl = hi + 3 * C::SB;
                float4 h4[4], l4[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int r = 4 * a + i;
                    const int off = blk * (BS * 128) + r * 128 + ((bcol ^ (r & 7)) << 4);
                    const float4 x = *reinterpret_cast<const float4 *>(hi + off);
                    h4[i] = make_float4(__uint_as_float(hi_bits(x.x)), __uint_as_float(hi_bits(x.y)),
                                        __uint_as_float(hi_bits(x.z)), __uint_as_float(hi_bits(x.w)));
                    l4[i] = make_float4(x.x - h4[i].x, x.y - h4[i].y, x.z - h4[i].z, x.w - h4[i].w);
                    *reinterpret_cast<float4 *>(hi + off) = h4[i];
                    *reinterpret_cast<float4 *>(lo + off) = l4[i];
                }
                if (KIND == 0 || part == 0) {
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const int col = 32 * blk + 4 * bcol + c;
                        const int toff = col * 128 + ((a ^ (col & 7)) << 4);
                        *reinterpret_cast<float4 *>(th + toff) =
                            make_float4(f4_at(h4[0], c), f4_at(h4[1], c), f4_at(h4[2], c), f4_at(h4[3], c));
                        *reinterpret_cast<float4 *>(tl + toff) =
                            make_float4(f4_at(l4[0], c), f4_at(l4[1], c), f4_at(l4[2], c), f4_at(l4[3], c));
                    }
                }
            }
            fence_async_smem();
            mbar_arrive(BAR(B_SS + st));
        }
    } else if (warp >= 8) {
        // ------------------------------------------------------------ elementwise
        regs_inc<256>();
        const int quad = warp & 3;
        const int row = quad * 32 + lane;            // TMEM lane = row of the fixed tile
        const uint32_t lb = (uint32_t)(quad * 32) << 16;
        const long long bh = ((long long)b * p.H + h) * p.T;
        const int grow_ = fixed * BT + row;          // global index of this thread's fixed row
        float my_nl2 = 0.f, my_ndd = 0.f;            // dq: this query row's -lse2 and -D / sqrt(d)
        if (KIND == 1 && grow_ < p.T) {
            my_nl2 = -__ldg(p.lse2 + bh + grow_);
            my_ndd = -__ldg(p.dvec + bh + grow_) * p.ds_scale;
        }
        const uint64_t scale2 = f2(p.scale_log2, p.scale_log2), ds2 = f2(p.ds_scale, p.ds_scale);
        constexpr int NA = KIND == 0 ? 2 : 1;        // accumulators: dkdv dV, dK; dq dQ
        float rs[NA][D];                             // this row's running sums
#pragma unroll
        for (int a = 0; a < NA; a++)
#pragma unroll
            for (int c = 0; c < D; c++) rs[a][c] = 0.f;
        bool ok = true;
        for (int it = 0; it < count; it++) {
            const int tcol = first + it;             // streamed tile index
            const int xb = it & 1;                   // X/Y buffer
            float *st_l = stats + (it & 1) * 2 * BS;   // dkdv: -lse2 and -D/sqrt(d) of the 32 query columns
            if (KIND == 0) {
                if (row < BS) {
                    const int q = tcol * BS + row;
                    st_l[row] = q < p.T ? -__ldg(p.lse2 + bh + q) : 0.f;
                    st_l[BS + row] = q < p.T ? -__ldg(p.dvec + bh + q) * p.ds_scale : 0.f;
                }
                mbar_arrive(BAR(B_ST));
                if (!(ok = wait_w(B_ST, it, 0x543))) break;
            }
            if (!(ok = wait_w(B_XY + xb, it >> 1, 0x541))) break;
            tc_fence_after();
            const uint32_t tX = tmem + lb + xy_col<D>(xb, 0), tY = tmem + lb + xy_col<D>(xb, 1);
            const uint32_t tW1L = tmem + lb + xy_col<D>(xb, 2), tW2L = tmem + lb + xy_col<D>(xb, 3);
            // P = 2^(X scale - lse2), dS = P (Y - D) / sqrt(d), on f32x2 pairs; the
            // causal and past-T masks only in tiles that reach them.  16 columns
            // at a time (all X/Y reads of a half complete before its P/dS high
            // parts overwrite them).
            const bool need_mask = KIND == 0 ? (tcol * BS < fixed * BT + BT - 1 || (tcol + 1) * BS > p.T)
                                             : ((tcol + 1) * BS - 1 > fixed * BT);
            auto tile = [&](auto masked_tag) {
                constexpr bool MASKED = decltype(masked_tag)::value;
#pragma unroll
                for (int h2 = 0; h2 < 2; h2++) {
                    uint32_t xs[16], ys[16];
                    tmem_ld16(tX + 16 * h2, xs);
                    tmem_ld16(tY + 16 * h2, ys);
                    tmem_wait_ld();
                    // P first (its parts stored while Y is still in registers), then dS
                    float pv[16];
#pragma unroll
                    for (int c = 0; c < 16; c += 2) {
                        const int cc = 16 * h2 + c;
                        const uint64_t nl2 = KIND == 0 ? *reinterpret_cast<const uint64_t *>(st_l + cc)   // query columns
                                                       : f2(my_nl2, my_nl2);                              // this query row
                        f2_split(fma2(f2(__uint_as_float(xs[c]), __uint_as_float(xs[c + 1])), scale2, nl2), pv[c],
                                 pv[c + 1]);
                        pv[c] = ex2(pv[c]);
                        pv[c + 1] = ex2(pv[c + 1]);
                        if (MASKED) {
#pragma unroll
                            for (int u = 0; u < 2; u++) {
                                const int sidx = tcol * BS + cc + u;   // streamed row (dkdv: query, dq: key)
                                if (KIND == 0 ? (sidx < grow_ || sidx >= p.T) : (sidx > grow_)) pv[c + u] = 0.f;
                            }
                        }
                    }
                    if (KIND == 0) {
                        uint32_t ph[16], pl[16];
#pragma unroll
                        for (int c = 0; c < 16; c++) {
                            ph[c] = hi_bits(pv[c]);
                            pl[c] = __float_as_uint(pv[c] - __uint_as_float(ph[c]));
                        }
                        tmem_st16(tX + 16 * h2, ph);
                        tmem_st16(tW1L + 16 * h2, pl);
                    }
                    uint32_t dh[16], dl[16];
#pragma unroll
                    for (int c = 0; c < 16; c += 2) {
                        const int cc = 16 * h2 + c;
                        const uint64_t ndd = KIND == 0 ? *reinterpret_cast<const uint64_t *>(st_l + BS + cc)
                                                       : f2(my_ndd, my_ndd);
                        const uint64_t t2 = fma2(f2(__uint_as_float(ys[c]), __uint_as_float(ys[c + 1])), ds2, ndd);
                        float dv[2];
                        f2_split(fma2(f2(pv[c], pv[c + 1]), t2, 0ull), dv[0], dv[1]);
                        if (MASKED) {
                            // query 0 attends to key 0 alone: P = 1 and dS = dP - D = 0
                            // exactly (train.c:393-400 forms the row dot from P and dP,
                            // so it gets the exact zero; D = dO . O from the pre-pass
                            // would leave the products' 1e-7)
#pragma unroll
                            for (int u = 0; u < 2; u++)
                                if (KIND == 0 ? tcol * BS + cc + u == 0 : grow_ == 0) dv[u] = 0.f;
                        }
#pragma unroll
                        for (int u = 0; u < 2; u++) {
                            dh[c + u] = hi_bits(dv[u]);
                            dl[c + u] = __float_as_uint(dv[u] - __uint_as_float(dh[c + u]));
                        }
                    }
                    tmem_st16(tY + 16 * h2, dh);
                    tmem_st16(tW2L + 16 * h2, dl);
                }
            };
            if (need_mask) tile(std::true_type{});
            else tile(std::false_type{});
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(BAR(B_W + xb));
            if (it % kGroup == kGroup - 1 || it == count - 1) {
                // the group's sums (complete with this tile's accumulation) -> the
                // running sums, then the accumulators are free for the next group
                if (!(ok = wait_w(B_ACC + xb, it >> 1, 0x545))) break;
                tc_fence_after();
#pragma unroll
                for (int a = 0; a < NA; a++) {
#pragma unroll
                    for (int c0 = 0; c0 < D; c0 += 16) {
                        uint32_t acc[16];
                        tmem_ld16(tmem + lb + (a ? C::TM_A2 : C::TM_A1) + c0, acc);
                        tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 16; c++) rs[a][c0 + c] += __uint_as_float(acc[c]);
                    }
                }
                tc_fence_before();
                mbar_arrive(BAR(B_AF));
            }
        }
        // epilogue: running sums -> global (fp32, optionally added to the output)
        if (__all_sync(0xffffffffu, ok && count > 0) && grow_ < p.T) {
#pragma unroll
            for (int a = 0; a < NA; a++) {
                // dkdv: a=0 -> dV (out2), a=1 -> dK (out1);  dq: dQ (out1)
                float *outp = KIND == 0 ? (a == 0 ? p.out2 : p.out1) : p.out1;
                float *dst = outp + ((long long)b * p.T + grow_) * p.out_stride + (long long)h * D;
#pragma unroll
                for (int c = 0; c < D; c += 4) {
                    float4 v = make_float4(rs[a][c], rs[a][c + 1], rs[a][c + 2], rs[a][c + 3]);
                    float4 *d4 = reinterpret_cast<float4 *>(dst + c);
                    if (p.accumulate) {
                        const float4 o = *d4;
                        v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
                    }
                    *d4 = v;
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
        tmem_dealloc(tmem, C::TM_COLS);
    }
#undef BAR
}

}  // namespace fbt
}  // namespace attn

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace attn_host {

bool ensure_smem_attr(const void *func, size_t bytes);
int launch_bwd_rowdot(int dtype, int D, const void *o, const void *dout, const float *lse, float *ws,
                      long long in_stride, long long out_stride, int B, int H, int T, cudaStream_t s);

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn_bt() {
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

// 3-D view {columns, T, B} of a (B*T, stride) fp32 tensor; 32 x rows boxes
// (128 bytes wide) with the 128-byte swizzle.  Cached per (pointer, shape).
static bool map_f32_bt(CUtensorMap *m, const void *ptr, int cols, int T, int B, long long stride, int rows) {
    struct Entry { const void *ptr; int cols, T, B, rows; long long stride; CUtensorMap map; };
    static thread_local Entry cache[16];
    static thread_local int next = 0;
    for (auto &e : cache)
        if (e.ptr == ptr && e.cols == cols && e.T == T && e.B == B && e.rows == rows && e.stride == stride) {
            *m = e.map;
            return true;
        }
    auto fn = encode_fn_bt();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)stride * 4, (cuuint64_t)stride * 4 * T};
    cuuint32_t box[3] = {32, (cuuint32_t)rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    if (fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void *>(ptr), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    cache[next] = Entry{ptr, cols, T, B, rows, stride, *m};
    next = (next + 1) % 16;
    return true;
}

bool bwd_tf32_sm100_supported(int D, long long in_stride, long long out_stride) {
    return (D == 32 || D == 64) && in_stride % 4 == 0 && out_stride % 4 == 0 && encode_fn_bt() != nullptr;
}

template <int D>
static int launch_bwd_tf32_t(const void *dout, const void *q, const void *k, const void *v, const void *o,
                             const float *lse, void *dq, void *dk, void *dv, int accumulate, void *ws,
                             long long in_stride, long long out_stride, int B, int H, int T, int *err,
                             cudaStream_t s) {
    using namespace attn::fbt;
    int st = launch_bwd_rowdot(ATTN_F32, D, o, dout, lse, static_cast<float *>(ws), in_stride, out_stride, B, H,
                               T, s);
    if (st) return st;
    CUtensorMap mq, mk, mv, mdo, mq32, mk32, mv32, mdo32;
    if (!map_f32_bt(&mq, q, H * D, T, B, in_stride, BT) || !map_f32_bt(&mk, k, H * D, T, B, in_stride, BT) ||
        !map_f32_bt(&mv, v, H * D, T, B, in_stride, BT) || !map_f32_bt(&mdo, dout, H * D, T, B, in_stride, BT) ||
        !map_f32_bt(&mq32, q, H * D, T, B, in_stride, BS) || !map_f32_bt(&mk32, k, H * D, T, B, in_stride, BS) ||
        !map_f32_bt(&mv32, v, H * D, T, B, in_stride, BS) || !map_f32_bt(&mdo32, dout, H * D, T, B, in_stride, BS))
        return set_error(ATTN_ERR_CUDA, "3xTF32 backward: cuTensorMapEncodeTiled failed");
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
    const size_t smem = Cfg<D>::SMEM;
    if (!ensure_smem_attr((const void *)bwd_tf32_kernel<D, 0>, smem) ||
        !ensure_smem_attr((const void *)bwd_tf32_kernel<D, 1>, smem))
        return set_error(ATTN_ERR_CUDA, "3xTF32 backward: cannot set shared-memory size");
    const int n_ft = (T + BT - 1) / BT;
    const long long n_units = (long long)B * H * n_ft;
    if (n_units > (1LL << 30)) return set_error(ATTN_ERR_INVALID, "3xTF32 backward: too many tiles");
    const dim3 grid((unsigned)n_units);
    p.out1 = static_cast<float *>(dk);
    p.out2 = static_cast<float *>(dv);
    // fixed K, V; streamed Q, dO
    if ((st = check_pdl(launch_pdl(bwd_tf32_kernel<D, 0>, grid, dim3(kThreads), smem, s, mk, mv, mq32, mdo32, p),
                        "3xTF32 backward dkdv kernel")))
        return st;
    p.out1 = static_cast<float *>(dq);
    p.out2 = nullptr;
    // fixed Q, dO; streamed K, V
    return check_pdl(launch_pdl(bwd_tf32_kernel<D, 1>, grid, dim3(kThreads), smem, s, mq, mdo, mk32, mv32, p),
                     "3xTF32 backward dq kernel");
}

int launch_bwd_tf32_sm100(int D, const void *dout, const void *q, const void *k, const void *v, const void *o,
                          const float *lse, void *dq, void *dk, void *dv, int accumulate, void *ws,
                          long long in_stride, long long out_stride, int B, int H, int T, int *err,
                          cudaStream_t s) {
    if (((uintptr_t)dout | (uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)dq | (uintptr_t)dk |
         (uintptr_t)dv) & 15)
        return set_error(ATTN_ERR_INVALID, "3xTF32 backward: tensors must be 16-byte aligned");
    switch (D) {
        case 32: return launch_bwd_tf32_t<32>(dout, q, k, v, o, lse, dq, dk, dv, accumulate, ws, in_stride,
                                              out_stride, B, H, T, err, s);
        case 64: return launch_bwd_tf32_t<64>(dout, q, k, v, o, lse, dq, dk, dv, accumulate, ws, in_stride,
                                              out_stride, B, H, T, err, s);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "3xTF32 backward: head_dim %d", D);
    }
}

}  // namespace attn_host
