// decode_i8mma.cu -- KV-cached decode attention over an INT8 cache with the
// code dot products on the tensor cores (tcgen05.mma kind::i8, sm_100a).
//
// Semantics: cached_attention, transformer.c:203-248 -- for every head, one
// query row scores cache rows 0..len-1 with (q . k_j) / sqrt(d), softmaxes
// them and sums the value rows.  INT8 caches hold codes plus a per-(row, head)
// fp32 scale (the absmax scheme of gemm_bench.c:225-236); attention runs over
// the dequantised values code * scale.
//
// The SIMT streaming kernel spends ~2 instructions per cache byte turning
// codes into floats; here the codes never leave the integer domain.  Both
// products are exact integer matrix products on the tensor core, with the
// floating-point operand written as a 28-bit fixed-point number split into
// four 7-bit digits (each a signed byte):
//   scores   D_S[t][n] = sum_c Kcode[t][c] * qdigit[n][c]      M = 128 tokens, N = 8, K = 128 codes
//   values   D_O[c][n] = sum_t Vcode[t][c] * wdigit[n][t]      M = 128 codes (MN-major), N = 8, K = 128 tokens
// A cache row of H*D = 1024 codes is cut into eight 128-byte column blocks
// (two heads of d 64, or one head of d 128); every MMA works on one block, so
// an N = 8 operand holds four digits of each of the block's heads, and the
// int32 sums stay exact (|D_S| < 2^21, |D_O| < 2^21 per 128-row tile).
//
// Work split: the sequences' rows, concatenated, are cut into one equal
// range per CTA (so every SM streams the same number of bytes, whatever the
// lengths); a piece is the part of one sequence inside one CTA's range (all
// heads), and a CTA's pieces form one stream of 128-row tiles.  Per tile, the softmax warpgroups (one thread per token) turn the
// score digit sums into base-2 logits x, take the tile maxima of x and of the
// weight logits x + log2|vscale| over the warpgroup, fold the tile into the
// running (max, sum) per head, and write each token's weight
// w = 2^(x - max) * vscale as 28-bit fixed point relative to the tile's
// largest weight; after the value product they read the tile's sums out of
// TMEM and fold them into the output accumulators (online softmax over
// tiles).  The tensor core runs the score tile after the current one while
// the warpgroups work on the current weights, so the code stream never waits
// for them.  A piece ends with its output (one-piece sequence) or its
// partial (max, sum, unnormalised output) for the merge kernel.
// Roles: warp 0 streams code tiles (TMA, 128-byte swizzle) into an 8-stage
// ring, the scale tiles into a 2-stage ring and each piece's query row; warp
// 1 issues the MMAs (elected lane); warps 4-7 and 8-11 are two softmax
// warpgroups, each owning half of the heads (TMEM lane quadrant = warp & 3).
// Every mbarrier wait is bounded; a timeout records a code in the device
// error word and raises a CTA-wide abort flag.  No TMA multicast.
#include <algorithm>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "decode_launch.cuh"
#include "sm100.cuh"

namespace attn {
namespace dq {

using namespace sm100;

constexpr int TT = 128;                 // tokens per tile (TMEM lanes of the score products)
constexpr int NB = 8;                   // 128-byte column blocks per cache row (H * D = 1024)
constexpr int HD = NB * 128;            // codes per cache row
constexpr int KS = 8;                   // code-tile ring stages
constexpr int QN = 4;                   // piece-descriptor queue slots
constexpr int kThreads = 384;              // warp 0 TMA, warp 1 MMA, warps 4-11 softmax
constexpr int kMaxSeq = 1024;           // sequences per call (row table in shared memory)
constexpr int kMaxGrid = 160;           // CTAs at most (>= the SM count of a B200)
constexpr int TILE = TT * 128;          // bytes of one code tile: 128 tokens x 128 codes
constexpr int TM_COLS = 256;            // D_S and D_O double buffers (4 x 64 columns)
constexpr int TM_O = 128;

struct Params {
    const float *q;
    const int *lens;
    float *out;
    float *part_o;                      // [n_items][HD]
    float *part_ml;                     // [n_items][H][2]
    int *starts;                        // [n_seq + 1] first row of each sequence (rows concatenated)
    int *err;
    int n_seq, max_len, grid;           // partials: slot cta + sequence (< grid + n_seq)
    float qscale;                       // log2(e) / sqrt(D)
};

template <int D>
struct Geo {
    static constexpr int H = HD / D;
    static constexpr int HB = 128 / D;                  // heads per column block
    static constexpr int HW = H / 2;                    // heads per softmax warpgroup
    static constexpr int BW = NB / 2;                   // column blocks per softmax warpgroup
    static constexpr int SC = TT * H * 4;               // one tile of K (or V) scales
    static constexpr int OFF_RING = 0;
    static constexpr int OFF_QD = OFF_RING + KS * TILE;          // [2][NB] x 1 KB query digits
    static constexpr int OFF_W = OFF_QD + 2 * NB * 1024;          // [2][NB] x 1 KB weight digits
    static constexpr int OFF_SC = OFF_W + 2 * NB * 1024;          // [2 stages][K, V] scale tiles
    static constexpr int OFF_Q = OFF_SC + 4 * SC;                 // [2][HD] query rows
    static constexpr int OFF_RED = OFF_Q + 2 * HD * 4;            // [2 wg][2 parity][4 warps][HW][2]
    static constexpr int OFF_REDQ = OFF_RED + 2 * 2 * 4 * HW * 2 * 4;   // [2 wg][4 warps][BW] query maxima
    static constexpr int OFF_TAB = OFF_REDQ + 2 * 4 * BW * 4;     // lens, first rows
    static constexpr int OFF_PQ = OFF_TAB + (2 * kMaxSeq + 1) * 4;   // [QN][4] piece descriptors
    static constexpr int OFF_BAR = (OFF_PQ + QN * 16 + 7) / 8 * 8;
    static constexpr int B_FULL = 0, B_EMPTY = KS, B_SCF = 2 * KS, B_SCE = B_SCF + 2, B_SF = B_SCF + 4,
                         B_SE = B_SCF + 6, B_QF = B_SCF + 8, B_QE = B_SCF + 10, B_WR = B_SCF + 12,
                         B_OF = B_SCF + 14, B_OE = B_SCF + 16, B_SY = B_SCF + 18, B_PQF = B_SCF + 20,
                         B_PQE = B_PQF + QN, B_QR = B_PQE + QN, N_BAR = B_QR + 1;
    static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;          // abort flag, TMEM base
    static constexpr int SMEM = OFF_MISC + 16 + 1024;             // + alignment of the base
    static_assert(HB * D == 128 && HB * 4 <= 8, "block layout: four digits per head, 8 columns per block");
    static_assert(SMEM <= 232448, "shared memory");
};

// tcgen05 instruction descriptor, kind::i8: D int32 (bits 4-5 = 2), A and B
// signed 8-bit (bits 7-9, 10-12 = 1), majors in bits 15/16, N >> 3 in bits
// 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N, int a_mn_major, int b_mn_major) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// D[tmem] (+)= A[smem] * B[smem], signed 8-bit inputs, int32 accumulate (K = 32 per instruction)
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                 ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// byte offset of element (row r, byte k) in a tile of 128-byte rows stored
// with the 128-byte swizzle (16-byte chunk index XOR row mod 8)
__device__ __forceinline__ uint32_t swz(int r, int k) {
    return (uint32_t)(r * 128 + ((((k >> 4) ^ r) & 7) << 4) + (k & 15));
}
// digit sums d[0..3] (weights 2^0, 2^7, 2^14, 2^21) back to one float
__device__ __forceinline__ float undigit(const uint32_t *d) {
    return fmaf(fmaf(fmaf((float)(int)d[3], 128.f, (float)(int)d[2]), 128.f, (float)(int)d[1]), 128.f,
                (float)(int)d[0]);
}
__device__ __forceinline__ float pow2i(int e) { return __int_as_float((e + 127) << 23); }   // e in [-126, 127]
// order-preserving map of a float onto a signed int (for integer max reductions)
__device__ __forceinline__ int f2o(float f) {
    const int b = __float_as_int(f);
    return b ^ ((b >> 31) & 0x7fffffff);
}
__device__ __forceinline__ float o2f(int o) { return __int_as_float(o ^ ((o >> 31) & 0x7fffffff)); }

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
decode_i8mma_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                    const __grid_constant__ CUtensorMap tk32, const __grid_constant__ CUtensorMap tv32,
                    const __grid_constant__ CUtensorMap tks, const __grid_constant__ CUtensorMap tvs,
                    const __grid_constant__ Params p)
{
    pdl_begin();   // launched by launch_pdl
    using G = Geo<D>;
    constexpr int H = G::H, HB = G::HB, HW = G::HW, BW = G::BW;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *sb = smem_raw + (base - raw);
    int *lens_s = reinterpret_cast<int *>(sb + G::OFF_TAB);
    int *start_s = lens_s + kMaxSeq;
    volatile int *pqs = reinterpret_cast<volatile int *>(sb + G::OFF_PQ);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sb + G::OFF_MISC);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sb + G::OFF_MISC + 8);
    auto BAR = [&](int i) { return base + G::OFF_BAR + 8u * (uint32_t)i; };
    auto wait = [&](int b, uint32_t parity, int code) -> bool {
        return __all_sync(0xffffffffu, mbar_wait(BAR(b), parity & 1u, abort_flag, p.err, code));
    };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < KS; s++) {
            mbar_init(BAR(G::B_FULL + s), 1);
            mbar_init(BAR(G::B_EMPTY + s), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(BAR(G::B_SCF + i), 1);
            mbar_init(BAR(G::B_SCE + i), 256);
            mbar_init(BAR(G::B_SF + i), 1);
            mbar_init(BAR(G::B_SE + i), 256);
            mbar_init(BAR(G::B_QF + i), 1);
            mbar_init(BAR(G::B_QE + i), 256);
            mbar_init(BAR(G::B_WR + i), 256);
            mbar_init(BAR(G::B_OF + i), 1);
            mbar_init(BAR(G::B_OE + i), 256);
            mbar_init(BAR(G::B_SY + i), 128);       // one per softmax warpgroup
        }
        for (int i = 0; i < QN; i++) {
            mbar_init(BAR(G::B_PQF + i), 1);
            mbar_init(BAR(G::B_PQE + i), 9);        // the MMA warp and the eight softmax warps
        }
        mbar_init(BAR(G::B_QR), 256);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TM_COLS);
        tmem_relinquish();
    }
    // digit operands start as zeros: rows no head writes (d 128: rows 4-7) stay zero
    for (int i = threadIdx.x; i < 4 * NB * 1024 / 16; i += kThreads)
        reinterpret_cast<uint4 *>(sb + G::OFF_QD)[i] = make_uint4(0, 0, 0, 0);
    // piece table: lengths (clamped; bad ones flagged), then their prefix sums of pieces
    for (int e = threadIdx.x; e < p.n_seq; e += kThreads) {
        int len = p.lens ? __ldg(p.lens + e) : p.max_len;
        if (len < 1 || len > p.max_len) {
            if (blockIdx.x == 0) atomicExch(p.err, 0x100 + (len < 1 ? 1 : 2));
            len = len < 1 ? 1 : p.max_len;
        }
        lens_s[e] = len;
    }
    fence_async_smem();
    __syncthreads();
    if (warp == 0) {
        const int per = (p.n_seq + 31) / 32, e0 = lane * per, e1 = min(p.n_seq, e0 + per);
        int sum = 0;
        for (int e = e0; e < e1; e++) sum += lens_s[e];
        int incl = sum;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        int run = incl - sum;
        for (int e = e0; e < e1; e++) {
            start_s[e] = run;
            run += lens_s[e];
        }
        if (lane == 31) start_s[p.n_seq] = incl;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    asm volatile("griddepcontrol.launch_dependents;");   // the merge kernel may be scheduled
    // this CTA's rows [row0, row1) of the concatenated sequences
    const long long rows_all = start_s[p.n_seq];
    const int row0 = (int)(rows_all * blockIdx.x / gridDim.x), row1 = (int)(rows_all * (blockIdx.x + 1) / gridDim.x);
    if (blockIdx.x == 0)                            // row table for the merge kernel
        for (int e = threadIdx.x; e <= p.n_seq; e += kThreads) p.starts[e] = start_s[e];

    // The CTA's pieces form one stream of 128-row tiles.  Order of the
    // tensor-core work (and of the ring, which the loads follow):
    //   K(0), K(1), V(0), K(2), V(1), ..., K(last), V(last - 1), [next piece's K(0)], V(last), ...
    // so the score tile after the current one is always in flight while the
    // softmax warpgroups turn the current scores into weights.
    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tmap(&tk);
            prefetch_tmap(&tv);
            prefetch_tmap(&tk32);
            prefetch_tmap(&tv32);
            prefetch_tmap(&tks);
            prefetch_tmap(&tvs);
            int s = 0, use = 0, sc = 0, pq = 0;
            bool ok = true;
            // the eight code blocks of one tile; a tile with fewer than 128 rows
            // left in its piece loads only the 32-row boxes that hold them (the
            // rest of the stage keeps stale codes, which meet masked scores and
            // zero weights)
            auto load_codes = [&](bool vals, int y, int e, int rows) -> bool {
                const int nb = rows >= TT ? 1 : (rows + 31) / 32;
                const CUtensorMap *map = rows >= TT ? (vals ? &tv : &tk) : (vals ? &tv32 : &tk32);
                for (int b = 0; b < NB; b++) {
                    if (use >= KS && !mbar_wait(BAR(G::B_EMPTY + s), (uint32_t)(use / KS + 1) & 1u, abort_flag,
                                                p.err, 0x401))
                        return false;
                    const uint32_t dst = base + G::OFF_RING + s * TILE;
                    mbar_arrive_expect_tx(BAR(G::B_FULL + s), rows >= TT ? TILE : nb * 32 * 128);
                    for (int j = 0; j < nb; j++)
                        tma_load_3d(dst + j * 32 * 128, map, BAR(G::B_FULL + s), b * 128, y + j * 32, e);
                    s = (s + 1) % KS;
                    use++;
                }
                return true;
            };
            auto load_k = [&](int y, int e, int rows) -> bool {   // scales of the tile, then its eight K blocks
                const int ss = sc & 1;
                if (sc >= 2 &&
                    !mbar_wait(BAR(G::B_SCE + ss), (uint32_t)(sc / 2 + 1) & 1u, abort_flag, p.err, 0x403))
                    return false;
                const uint32_t sdst = base + G::OFF_SC + ss * 2 * G::SC;
                mbar_arrive_expect_tx(BAR(G::B_SCF + ss), 2 * G::SC);
                tma_load_3d(sdst, &tks, BAR(G::B_SCF + ss), 0, y, e);
                tma_load_3d(sdst + G::SC, &tvs, BAR(G::B_SCF + ss), 0, y, e);
                sc++;
                return load_codes(false, y, e, rows);
            };
            // the piece's descriptor into the queue and its query row into the
            // query buffer of its parity (pieces and queue entries count alike)
            auto publish = [&](int v, int e, int r0, int n) -> bool {
                const int q = pq % QN, qb = pq & 1;
                if (pq >= QN &&
                    !mbar_wait(BAR(G::B_PQE + q), (uint32_t)(pq / QN + 1) & 1u, abort_flag, p.err, 0x402))
                    return false;
                if (v >= 0) {
                    if (pq >= 2 &&
                        !mbar_wait(BAR(G::B_QE + qb), (uint32_t)(pq / 2 + 1) & 1u, abort_flag, p.err, 0x404))
                        return false;
                    mbar_arrive_expect_tx(BAR(G::B_QF + qb), HD * 4);
                    bulk_load(base + G::OFF_Q + qb * HD * 4, p.q + (long long)e * HD, HD * 4, BAR(G::B_QF + qb));
                }
                pqs[4 * q] = v;
                pqs[4 * q + 1] = e;
                pqs[4 * q + 2] = r0;
                pqs[4 * q + 3] = n;
                mbar_arrive(BAR(G::B_PQF + q));
                pq++;
                return true;
            };
            struct Piece { int v, e, r0, n, nt; };
            int e_cur = 0;                           // sequence holding row0
            {
                int lo = 0, hi = p.n_seq - 1;        // last e with start[e] <= row0
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (start_s[mid] <= row0) lo = mid; else hi = mid - 1;
                }
                e_cur = lo;
            }
            auto claim = [&]() -> Piece {            // the next piece of this CTA's range
                while (e_cur < p.n_seq) {
                    const int e = e_cur++;
                    const int a0 = max(row0, start_s[e]), a1 = min(row1, start_s[e + 1]);
                    if (a0 >= row1) break;
                    if (a1 > a0) {
                        const int n = a1 - a0;
                        return Piece{(int)blockIdx.x + e, e, a0 - start_s[e], n, (n + TT - 1) / TT};
                    }
                }
                e_cur = p.n_seq;
                return Piece{-1, 0, 0, 0, 0};
            };
            Piece cur = claim();
            if (cur.v >= 0) ok = publish(cur.v, cur.e, cur.r0, cur.n) && load_k(cur.r0, cur.e, cur.n);
            while (ok && cur.v >= 0) {
                Piece nxt{-1, 0, 0, 0, 0};
                for (int t = 0; ok && t < cur.nt; t++) {
                    if (t + 1 < cur.nt) {
                        ok = load_k(cur.r0 + (t + 1) * TT, cur.e, cur.n - (t + 1) * TT);
                    } else {
                        nxt = claim();
                        if (nxt.v >= 0) ok = publish(nxt.v, nxt.e, nxt.r0, nxt.n) && load_k(nxt.r0, nxt.e, nxt.n);
                    }
                    if (ok) ok = load_codes(true, cur.r0 + t * TT, cur.e, cur.n - t * TT);
                }
                cur = nxt;
            }
            if (ok) publish(-1, 0, 0, 0);            // end marker
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        const bool leader = elect_one();
        constexpr uint32_t idK = idesc_i8(TT, 8, 0, 0);     // K codes (K-major) x query digits (K-major)
        constexpr uint32_t idV = idesc_i8(128, 8, 1, 0);    // V codes (MN-major) x weight digits (K-major)
        int s = 0, use = 0, tk_n = 0, tv_n = 0, pq = 0, k = 0;
        bool ok = true;
        auto next_piece = [&](int &v, int &n) -> bool {   // descriptor of the next piece (v < 0: end)
            const int q = pq % QN;
            if (!wait(G::B_PQF + q, (uint32_t)(pq / QN), 0x411)) return false;
            v = pqs[4 * q];
            n = pqs[4 * q + 3];
            __syncwarp();
            if (leader) mbar_arrive(BAR(G::B_PQE + q));
            __syncwarp();
            pq++;
            return true;
        };
        // score tile: 8 blocks x 4 MMAs into D_S buffer (tk_n & 1); piece parity kp selects the query digits
        auto mma_k = [&](int kp) -> bool {
            const int buf = tk_n & 1;
            if (tk_n >= 2 && !wait(G::B_SE + buf, (uint32_t)((tk_n >> 1) + 1), 0x413)) return false;
            tc_fence_after();
            const uint32_t qd = base + G::OFF_QD + (kp & 1) * NB * 1024;
            for (int b = 0; b < NB; b++, use++, s = (s + 1) % KS) {
                if (!wait(G::B_FULL + s, (uint32_t)(use / KS), 0x414)) return false;
                tc_fence_after();
                if (leader) {
                    const uint32_t a = base + G::OFF_RING + s * TILE;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)          // 32 codes per step
                        mma_i8_ss(tmem + buf * 64 + 8 * b, sw128_desc(a + 32 * kk, 16, 1024),
                                  sw128_desc(qd + b * 1024 + 32 * kk, 16, 1024), idK, kk > 0);
                    mma_commit(BAR(G::B_EMPTY + s));
                }
                __syncwarp();
            }
            if (leader) mma_commit(BAR(G::B_SF + buf));
            __syncwarp();
            tk_n++;
            return true;
        };
        // value tile: 8 blocks x 4 MMAs into D_O buffer (tv_n & 1) from weight digits (tv_n & 1)
        auto mma_v = [&]() -> bool {
            const int buf = tv_n & 1;
            if (!wait(G::B_WR + buf, (uint32_t)(tv_n >> 1), 0x415)) return false;
            if (tv_n >= 2 && !wait(G::B_OE + buf, (uint32_t)((tv_n >> 1) + 1), 0x416)) return false;
            tc_fence_after();
            const uint32_t wd = base + G::OFF_W + buf * NB * 1024;
            for (int b = 0; b < NB; b++, use++, s = (s + 1) % KS) {
                if (!wait(G::B_FULL + s, (uint32_t)(use / KS), 0x417)) return false;
                tc_fence_after();
                if (leader) {
                    const uint32_t a = base + G::OFF_RING + s * TILE;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)          // 32 tokens (4 KB of the tile) per step
                        mma_i8_ss(tmem + TM_O + buf * 64 + 8 * b, sw128_desc(a + 4096 * kk, 16, 1024),
                                  sw128_desc(wd + b * 1024 + 32 * kk, 16, 1024), idV, kk > 0);
                    mma_commit(BAR(G::B_EMPTY + s));
                }
                __syncwarp();
            }
            if (leader) mma_commit(BAR(G::B_OF + buf));
            __syncwarp();
            tv_n++;
            return true;
        };
        int v = -1, n = 0;
        ok = next_piece(v, n);
        if (ok && v >= 0) ok = wait(G::B_QR, 0u, 0x412) && mma_k(0);
        while (ok && v >= 0) {
            const int nt = (n + TT - 1) / TT;
            int v2 = -1, n2 = 0;
            for (int t = 0; ok && t < nt; t++) {
                if (t + 1 < nt) {
                    ok = mma_k(k);
                } else {
                    ok = next_piece(v2, n2);
                    if (ok && v2 >= 0) ok = wait(G::B_QR, (uint32_t)(k + 1), 0x412) && mma_k(k + 1);
                }
                if (ok) ok = mma_v();
            }
            v = v2;
            n = n2;
            k++;
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ softmax warpgroups
        // warpgroup g (warps 4-7, 8-11) owns heads [g*HW, (g+1)*HW) = column
        // blocks [g*BW, (g+1)*BW); thread t is token t of a tile and code t of
        // a block (TMEM lane t, quadrant warp & 3)
        const int g = (warp - 4) >> 2, w4 = warp & 3;
        const int t = w4 * 32 + lane;
        const int half = t / D;                     // head of code t within its block
        const uint32_t tl = tmem + ((uint32_t)(w4 * 32) << 16);
        float *redq = reinterpret_cast<float *>(sb + G::OFF_REDQ) + g * 4 * BW;
        // per-warp partials exchanged at a warpgroup sync; two buffers by sync
        // parity, so a warp that runs ahead writes the other one
        float *red0 = reinterpret_cast<float *>(sb + G::OFF_RED) + g * 2 * 4 * HW * 2;
        int pq = 0, ts = 0, to = 0, sc = 0, sy = 0;   // queue entries, score tiles, value tiles, scale tiles, syncs
        bool ok = true;
        auto wg_sync = [&](int code) -> bool {
            mbar_arrive(BAR(G::B_SY + g));
            const bool r = wait(G::B_SY + g, (uint32_t)sy, code);
            sy++;
            return r;
        };
        auto next_piece = [&](int &v, int &e, int &n) -> bool {
            const int q = pq % QN;
            if (!wait(G::B_PQF + q, (uint32_t)(pq / QN), 0x421)) return false;
            v = pqs[4 * q];
            e = pqs[4 * q + 1];
            n = pqs[4 * q + 3];
            __syncwarp();
            if (lane == 0) mbar_arrive(BAR(G::B_PQE + q));
            __syncwarp();
            pq++;
            return true;
        };
        // query digits of piece k (its query row in buffer k & 1) for this
        // warpgroup's blocks; qs = qscale * 2^-e per head
        float qs[HW];
        auto query_step = [&](int k) -> bool {
            if (!wait(G::B_QF + (k & 1), (uint32_t)(k >> 1), 0x422)) return false;
            float qv[BW];
            const float *qrow = reinterpret_cast<const float *>(sb + G::OFF_Q + (k & 1) * HD * 4);
#pragma unroll
            for (int bl = 0; bl < BW; bl++) qv[bl] = qrow[(g * BW + bl) * 128 + t];
            mbar_arrive(BAR(G::B_QE + (k & 1)));
#pragma unroll
            for (int bl = 0; bl < BW; bl++) {
                const unsigned m = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(qv[bl])));
                if (lane == 0) redq[w4 * BW + bl] = __uint_as_float(m);
            }
            if (!wg_sync(0x423)) return false;
            int qe[BW];                             // this thread's fixed-point exponent per block
#pragma unroll
            for (int hl = 0; hl < HW; hl++) {
                const int bl = hl / HB, hh = hl % HB;
                float mq = 0.f;
#pragma unroll
                for (int w = 0; w < 4; w++)
                    if (HB == 1 || (w >> 1) == hh) mq = fmaxf(mq, redq[w * BW + bl]);
                // 2^e * max|q| < 2^27
                const int ex = mq > 0.f ? min(126, 153 - (int)((__float_as_uint(mq) >> 23) & 255)) : 0;
                qs[hl] = p.qscale * pow2i(-ex);
                if (HB == 1 || hh == half) qe[bl] = ex;
            }
            uint8_t *qd = sb + G::OFF_QD + (k & 1) * NB * 1024;
#pragma unroll
            for (int bl = 0; bl < BW; bl++) {
                const int Q = __float2int_rn(qv[bl] * pow2i(qe[bl]));
                const int mag = abs(Q), sg = Q < 0 ? -1 : 1;
#pragma unroll
                for (int d = 0; d < 4; d++)         // rows of the block's other head stay zero at this code
                    qd[(g * BW + bl) * 1024 + swz(4 * half + d, t)] = (uint8_t)(int8_t)(sg * ((mag >> (7 * d)) & 127));
            }
            fence_async_smem();
            mbar_arrive(BAR(G::B_QR));
            return true;
        };
        // per piece, per head: running max m (uniform over the warpgroup),
        // this thread's share of the sum, and the output accumulator of this
        // thread's code in each block; pending (alpha, scale) of the value
        // tile whose sums are not read out yet
        float mrun[HW], lsum[HW], pal[HW], psc[HW], oacc[BW];
        // scores of the next tile -> weights (digits into buffer ts & 1)
        auto softmax_tile = [&](int tt, int n) -> bool {
            const int ss = sc & 1, buf = ts & 1;
            if (!wait(G::B_SCF + ss, (uint32_t)(sc >> 1), 0x424)) return false;
            if (!wait(G::B_SF + buf, (uint32_t)(ts >> 1), 0x425)) return false;
            tc_fence_after();
            uint32_t dsum[32];
            tmem_ld32(tl + buf * 64 + 32 * g, dsum);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(BAR(G::B_SE + buf));
            const float *ksr = reinterpret_cast<const float *>(sb + G::OFF_SC + ss * 2 * G::SC) + t * H + g * HW;
            const float *vsr = ksr + G::SC / 4;
            const bool valid = tt * TT + t < n;
            float x[HW], xp[HW];
#pragma unroll
            for (int hl = 0; hl < HW; hl++) {
                x[hl] = valid ? undigit(dsum + 8 * (hl / HB) + 4 * (hl % HB)) * qs[hl] * ksr[hl] : -INFINITY;
                xp[hl] = valid ? x[hl] + __log2f(fabsf(vsr[hl])) : -INFINITY;
            }
            uint32_t neg = 0;
#pragma unroll
            for (int hl = 0; hl < HW; hl++) neg |= (vsr[hl] < 0.f ? 1u : 0u) << hl;
            mbar_arrive(BAR(G::B_SCE + ss));
            sc++;
            // tile maxima of the logits and of the weight logits over the warpgroup
            float *red = red0 + (sy & 1) * 4 * HW * 2;
#pragma unroll
            for (int hl = 0; hl < HW; hl++) {
                const int a = __reduce_max_sync(0xffffffffu, f2o(x[hl]));
                const int b = __reduce_max_sync(0xffffffffu, f2o(xp[hl]));
                if (lane == 0) {
                    reinterpret_cast<int *>(red)[(w4 * HW + hl) * 2] = a;
                    reinterpret_cast<int *>(red)[(w4 * HW + hl) * 2 + 1] = b;
                }
            }
            if (!wg_sync(0x426)) return false;
            uint8_t *wb = sb + G::OFF_W + buf * NB * 1024 + g * BW * 1024;
#pragma unroll
            for (int hl = 0; hl < HW; hl++) {
                int a = reinterpret_cast<const int *>(red)[hl * 2], b = reinterpret_cast<const int *>(red)[hl * 2 + 1];
#pragma unroll
                for (int w = 1; w < 4; w++) {
                    a = max(a, reinterpret_cast<const int *>(red)[(w * HW + hl) * 2]);
                    b = max(b, reinterpret_cast<const int *>(red)[(w * HW + hl) * 2 + 1]);
                }
                const float mx = o2f(a), xmt = o2f(b);
                const float mn = fmaxf(mrun[hl], mx);           // finite: every tile has a valid row
                const float alpha = ex2(mrun[hl] - mn);         // 0 on the piece's first tile
                lsum[hl] = lsum[hl] * alpha + ex2(x[hl] - mn);
                mrun[hl] = mn;
                pal[hl] = alpha;
                // weights 2^(xp - xmt) as 28-bit fixed point (a tile whose value
                // scales are all zero has xmt = -inf and all-zero weights)
                const bool any = xmt > -INFINITY;
                psc[hl] = any ? ex2(xmt - 27.f - mn) : 0.f;
                const int W = any ? __float2int_rn(ex2(xp[hl] - xmt + 27.f)) : 0;   // 0 .. 2^27
                const int sg = (neg >> hl) & 1 ? -1 : 1;
#pragma unroll
                for (int d = 0; d < 4; d++)
                    wb[(hl / HB) * 1024 + swz(4 * (hl % HB) + d, t)] = (uint8_t)(int8_t)(sg * ((W >> (7 * d)) & 127));
            }
            fence_async_smem();
            mbar_arrive(BAR(G::B_WR + buf));
            ts++;
            return true;
        };
        // value sums of the oldest pending tile -> output accumulators
        auto readout = [&]() -> bool {
            const int buf = to & 1;
            if (!wait(G::B_OF + buf, (uint32_t)(to >> 1), 0x427)) return false;
            tc_fence_after();
            uint32_t osum[32];
            tmem_ld32(tl + TM_O + buf * 64 + 32 * g, osum);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(BAR(G::B_OE + buf));
#pragma unroll
            for (int bl = 0; bl < BW; bl++) {
#pragma unroll
                for (int hh = 0; hh < HB; hh++) {
                    if (hh != half) continue;
                    const int hl = bl * HB + hh;
                    oacc[bl] = oacc[bl] * pal[hl] + undigit(osum + 8 * bl + 4 * hh) * psc[hl];
                }
            }
            to++;
            return true;
        };
        int v = -1, e = 0, n = 0;
        ok = next_piece(v, e, n);
        if (ok && v >= 0) ok = query_step(0);
        for (int k = 0; ok && v >= 0; k++) {
            const int nt = (n + TT - 1) / TT;
            const bool whole = n == lens_s[e];      // the sequence lies in this CTA's range
#pragma unroll
            for (int hl = 0; hl < HW; hl++) { mrun[hl] = -INFINITY; lsum[hl] = 0.f; }
#pragma unroll
            for (int bl = 0; bl < BW; bl++) oacc[bl] = 0.f;
            for (int tt = 0; ok && tt < nt; tt++) {
                if (tt > 0) {                       // pal/psc of tile tt-1 are consumed before softmax overwrites them
                    ok = readout();
                    if (!ok) break;
                }
                ok = softmax_tile(tt, n);
            }
            if (!ok) break;
            int v2 = -1, e2 = 0, n2 = 0;            // the next piece's query digits before this piece's last value tile
            if (!(ok = next_piece(v2, e2, n2))) break;
            if (v2 >= 0 && !(ok = query_step(k + 1))) break;
            if (!(ok = readout())) break;
            // sums over the warpgroup, then the piece's output or partial
            float *red = red0 + (sy & 1) * 4 * HW * 2;
#pragma unroll
            for (int hl = 0; hl < HW; hl++) {
                float l = lsum[hl];
#pragma unroll
                for (int off = 16; off >= 1; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
                if (lane == 0) red[(w4 * HW + hl) * 2] = l;
            }
            if (!(ok = wg_sync(0x428))) break;
            float L[HW];
#pragma unroll
            for (int hl = 0; hl < HW; hl++)
                L[hl] = red[hl * 2] + red[(HW + hl) * 2] + red[(2 * HW + hl) * 2] + red[(3 * HW + hl) * 2];
            float *dst = (whole ? p.out + (long long)e * HD : p.part_o + (long long)v * HD) + g * BW * 128 + t;
#pragma unroll
            for (int bl = 0; bl < BW; bl++) {
#pragma unroll
                for (int hh = 0; hh < HB; hh++) {
                    if (hh != half) continue;
                    const int hl = bl * HB + hh;
                    dst[bl * 128] = whole ? oacc[bl] / L[hl] : oacc[bl];
                }
            }
            if (!whole) {
#pragma unroll
                for (int hl = 0; hl < HW; hl++)
                    if (t == hl) {
                        p.part_ml[((long long)v * H + g * HW + hl) * 2] = mrun[hl];
                        p.part_ml[((long long)v * H + g * HW + hl) * 2 + 1] = L[hl];
                    }
            }
            v = v2;
            e = e2;
            n = n2;
        }
    }

    // ---------------------------------------------------------------- teardown
    tc_fence_before();
    __syncthreads();
    if (*abort_flag) {
        // let copies / MMAs already in flight drain before the CTA releases its memory
        for (int i = 0; i < 1000; i++) __nanosleep(1000);
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TM_COLS);
    }
}

// Sequences split over several CTAs' row ranges: combine the pieces' partial
// (max, sum, output) per head (base-2 maxima).  Grid (sequence, quarter of
// the row); the piece of sequence e in CTA c's range has slot c + e.  The
// per-(piece, head) factors 2^(m_i - M) / L are made once in shared memory,
// so each output is one pass of independent loads.
template <int D>
__global__ void __launch_bounds__(256)
decode_i8mma_merge(const __grid_constant__ Params p)
{
    constexpr int H = HD / D;
    __shared__ int slots[kMaxGrid];
    __shared__ float fac[kMaxGrid][H];
    __shared__ int n_slots;
    const int e = blockIdx.x;
    // launched as a programmatic dependent of the main kernel: its CTAs may start
    // on SMs the main kernel has left; the partials are read only after the main
    // grid completed and its writes are visible
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (threadIdx.x == 0) {
        const long long rows_all = p.starts[p.n_seq];
        const long long s0 = p.starts[e], s1 = p.starts[e + 1];
        auto first_row = [&](long long c) { return rows_all * c / p.grid; };
        long long c = s0 * p.grid / rows_all;       // CTA holding row s0 (adjusted for rounding)
        while (c + 1 < p.grid && first_row(c + 1) <= s0) c++;
        while (c > 0 && first_row(c) > s0) c--;
        int n = 0;
        for (long long lo = first_row(c); c < p.grid && lo < s1; c++) {
            const long long hi = first_row(c + 1);
            if (hi > (lo > s0 ? lo : s0)) slots[n++] = (int)c + e;   // rows of e in this range
            lo = hi;
        }
        n_slots = n;
    }
    __syncthreads();
    const int n = n_slots;
    if (n <= 1) return;                             // one range: written by the main kernel
    if (threadIdx.x < H) {
        const int h = threadIdx.x;
        float M = -INFINITY, L = 0.f;
        for (int i = 0; i < n; i++) M = fmaxf(M, p.part_ml[((long long)slots[i] * H + h) * 2]);
        for (int i = 0; i < n; i++) {
            const float f = ex2(p.part_ml[((long long)slots[i] * H + h) * 2] - M);
            fac[i][h] = f;
            L += p.part_ml[((long long)slots[i] * H + h) * 2 + 1] * f;
        }
        const float inv = 1.f / L;
        for (int i = 0; i < n; i++) fac[i][h] *= inv;
    }
    __syncthreads();
    const int x = blockIdx.y * 256 + threadIdx.x, h = x / D;
    float O = 0.f;
#pragma unroll 4
    for (int i = 0; i < n; i++) O += p.part_o[(long long)slots[i] * HD + x] * fac[i][h];
    p.out[(long long)e * HD + x] = O;
}

}  // namespace dq
}  // namespace attn

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace attn_host {

bool ensure_smem_attr(const void *func, size_t bytes);

static PFN_cuTensorMapEncodeTiled_v12000 i8_encode_fn() {
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

// 3-D view {cols, cap, n_seq} of a cache (codes: uint8, 128 x 128 boxes with
// the 128-byte swizzle; scales: fp32, cols x 128 boxes, no swizzle).  Rows past
// cap read as zeros.  Cached per (pointer, shape).
static bool i8_map(CUtensorMap *m, const void *ptr, bool codes, int cols, long long cap, int n_seq,
                   long long row_bytes, int box_rows = attn::dq::TT) {
    struct Entry { const void *ptr; bool codes; int cols; long long cap; int n_seq; long long rb; int br; CUtensorMap map; };
    static thread_local Entry cache[24];
    static thread_local int next = 0;
    for (auto &c : cache)
        if (c.ptr == ptr && c.codes == codes && c.cols == cols && c.cap == cap && c.n_seq == n_seq && c.rb == row_bytes &&
            c.br == box_rows) {
            *m = c.map;
            return true;
        }
    auto fn = i8_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)cap, (cuuint64_t)n_seq};
    cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)(row_bytes * cap)};
    cuuint32_t box[3] = {codes ? 128u : (cuuint32_t)cols, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, codes ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                    const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    codes ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    cache[next] = Entry{ptr, codes, cols, cap, n_seq, row_bytes, box_rows, *m};
    next = (next + 1) % 24;
    return true;
}

bool decode_i8mma_shape_ok(int heads, int head_dim, int kv_dtype) {
    return kv_dtype == ATTN_I8 && (long long)heads * head_dim == attn::dq::HD && (head_dim == 64 || head_dim == 128);
}

bool decode_i8mma_ok(const DecodeLaunch &L) {
    if (!decode_i8mma_shape_ok(L.heads, L.head_dim, L.kv_dtype) || L.kptrs || L.n_seq > attn::dq::kMaxSeq)
        return false;
    if (L.row_stride % 16 || L.row_stride < attn::dq::HD) return false;
    if (((uintptr_t)L.kbase | (uintptr_t)L.vbase | (uintptr_t)L.ksbase | (uintptr_t)L.vsbase | (uintptr_t)L.q) & 15)
        return false;
    if (L.cap > (1LL << 31) || (long long)L.max_len * L.n_seq >= (1LL << 31)) return false;   // int row indices
    return i8_encode_fn() != nullptr;
}

// Workspace: the row table, then one partial (max and sum per head, output
// row) per slot cta + sequence.
size_t decode_i8mma_ws_bytes(int n_seq, int heads, int head_dim, int max_len) {
    (void)max_len;
    const long long slots = (long long)attn::dq::kMaxGrid + n_seq;
    size_t r = ((size_t)(n_seq + 1) * sizeof(int) + 255) / 256 * 256;
    r += ((size_t)slots * heads * 2 * sizeof(float) + 255) / 256 * 256;           // part_ml
    r += ((size_t)slots * heads * head_dim * sizeof(float) + 255) / 256 * 256;    // part_o
    return r;
}

template <int D>
static int launch_i8mma_t(const DecodeLaunch &L) {
    using namespace attn::dq;
    using Gm = Geo<D>;
    Params p;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    p.grid = std::max(1, std::min(sms, kMaxGrid));
    p.n_seq = L.n_seq;
    p.max_len = L.max_len;
    const long long slots = (long long)kMaxGrid + L.n_seq;
    char *ws = static_cast<char *>(L.ws);
    const size_t t_bytes = ((size_t)(L.n_seq + 1) * sizeof(int) + 255) / 256 * 256;
    const size_t ml_bytes = ((size_t)slots * Gm::H * 2 * sizeof(float) + 255) / 256 * 256;
    p.starts = reinterpret_cast<int *>(ws);
    p.part_ml = reinterpret_cast<float *>(ws + t_bytes);
    p.part_o = reinterpret_cast<float *>(ws + t_bytes + ml_bytes);
    CUtensorMap mk, mv, mk32, mv32, mks, mvs;
    if (!i8_map(&mk, L.kbase, true, HD, L.cap, L.n_seq, L.row_stride) ||
        !i8_map(&mv, L.vbase, true, HD, L.cap, L.n_seq, L.row_stride) ||
        !i8_map(&mk32, L.kbase, true, HD, L.cap, L.n_seq, L.row_stride, 32) ||
        !i8_map(&mv32, L.vbase, true, HD, L.cap, L.n_seq, L.row_stride, 32) ||
        !i8_map(&mks, L.ksbase, false, Gm::H, L.cap, L.n_seq, (long long)Gm::H * 4) ||
        !i8_map(&mvs, L.vsbase, false, Gm::H, L.cap, L.n_seq, (long long)Gm::H * 4))
        return set_error(ATTN_ERR_CUDA, "decode: cannot encode the cache tensor maps");
    p.q = L.q;
    p.lens = L.lens;
    p.out = L.out;
    p.err = L.err;
    p.qscale = attn::kLog2e / sqrtf((float)D);
    const size_t smem = Gm::SMEM;
    if (!ensure_smem_attr((const void *)decode_i8mma_kernel<D>, smem))
        return set_error(ATTN_ERR_CUDA, "decode: cannot set shared-memory size");
    int st = check_pdl(launch_pdl(decode_i8mma_kernel<D>, dim3(p.grid), dim3(kThreads), smem, L.stream, mk, mv, mk32,
                                  mv32, mks, mvs, p),
                       "decode_i8mma_kernel");
    if (st) return st;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(L.n_seq, HD / 256);
    lc.blockDim = dim3(256);
    lc.stream = L.stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    const cudaError_t ce = cudaLaunchKernelEx(&lc, decode_i8mma_merge<D>, p);
    if (ce != cudaSuccess) return set_error(ATTN_ERR_CUDA, "decode: merge launch: %s", cudaGetErrorString(ce));
    return check_launch("decode_i8mma_merge");
}

int launch_decode_i8mma(const DecodeLaunch &L) {
    switch (L.head_dim) {
        case 64: return launch_i8mma_t<64>(L);
        case 128: return launch_i8mma_t<128>(L);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "decode: no tensor-core INT8 kernel for this shape");
    }
}

}  // namespace attn_host
