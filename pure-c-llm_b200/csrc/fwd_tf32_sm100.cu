// fwd_tf32_sm100.cu -- causal flash forward for fp32 tensors on the Blackwell
// tensor cores with 3xTF32 products (sm_100a).
//
// Semantics: attention_forward, train.c:339-370, fp32 in and out.  Every
// product of two fp32 values x * y is formed as xh*yh + xh*yl + xl*yh, where
// xh is x with its 13 low mantissa bits cleared (exactly representable in
// tf32, so the MMA's operand conversion leaves it unchanged) and xl = x - xh
// (exact in fp32); the dropped xl*yl term and the tf32 view of the low parts
// are ~2^-21 relative.  Scores, exponentials (MUFU ex2, no polynomial), sums
// and accumulators are fp32, so results track the fp32 reference to ~1e-6.
//
// Persistent kernel, one query tile (128 rows) of one (batch, head) per work
// item, items dealt longest-first to the CTAs (LPT); key tiles of 64 rows.
// 12 warps per CTA:
//   warp 0      TMA producer: the raw fp32 Q tile into the Q-high buffer, raw
//               K and V tiles into the high halves of a 2-stage ring
//   warp 1      S issuer: S = Qh Kh^T + Qh Kl^T + Ql Kh^T, M=128, N=64, K=8,
//               tcgen05.mma kind::tf32, into one of two S buffers in TMEM
//   warp 2      PV issuer: O += Ph Vh + Ph Vl + Pl Vh (P from TMEM)
//   warp 3      spare
//   warps 4-7   splitters: clear the low bits of each landed Q and K tile in
//               place and write its low part next to it; write V transposed
//               (V^T, K-major, so that PV's B operand is K-major) as high and
//               low parts; then fence for the MMAs
//   warps 8-11  softmax: a thread owns one query row (one TMEM lane), reads
//               its S row, keeps the running max (rescaling O only when it
//               grows by more than 2^8) and sum, and writes P's high part over
//               the S row it read and P's low part to a separate TMEM block
// TMEM (d 32: 256 columns): S/Ph buffers [0,64) and [64,128), Pl [128,192),
// O [192, 192+D).  An S buffer is reused once the PV that read its P finished.
// Head dims 64 and up: the split query tile lives in TMEM (Qh in columns
// [0,D), Ql in [D,2D); the S products read their A operand from TMEM, so the
// tensor core does not re-read it from shared memory for every key tile), and
// the splitters move each landed query tile from its shared-memory staging
// buffer into TMEM (512 columns: Q parts, two S buffers, Pl, O, running O).
// At d 96 and 128 the split tile would not fit in shared memory next to a
// two-stage ring anyway; there key tiles are 32 rows.
// Every mbarrier wait is bounded; a timeout records a code in the device
// error word, raises a CTA-wide abort flag, and all roles fall through to the
// teardown, which frees TMEM.
#include "common.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <cudaTypedefs.h>
#include <functional>
#include <queue>
#include <vector>

namespace attn {
namespace ftf {

using namespace sm100;

constexpr int BM = 128;            // query rows per tile (TMEM lanes)
constexpr int kThreads = 384;
constexpr int kMaxCtas = 320;
constexpr int kMaxItems = 32768;
constexpr int kLocalItems = 256;
constexpr int kFold = 4;           // key tiles per fresh PV sum (see Cfg)

#ifndef ATTN_TF32_QT_MIN_D
#define ATTN_TF32_QT_MIN_D 64
#endif
template <int D>
struct Cfg {
    static constexpr bool QT = D >= ATTN_TF32_QT_MIN_D;   // query parts in TMEM
    static constexpr int BN = D > 64 ? 32 : 64;     // keys per tile
    static constexpr int CH = D / 32;               // 128-byte column chunks of a row
    static constexpr int QB = BM * D * 4;           // one fp32 Q tile (high or low part)
    static constexpr int KB = BN * D * 4;           // one fp32 K or V tile
    static constexpr int OFF_QH = 0, OFF_QL = QB;   // (TMEM mode: OFF_QH is the raw staging tile)
    static constexpr int OFF_ST = QT ? QB : 2 * QB; // stages: Kh, Kl, V raw then V^T low, V^T high
    static constexpr int STAGE = 4 * KB;
    static constexpr int OFF_BAR = OFF_ST + 2 * STAGE;
    static constexpr int OFF_ITEMS = OFF_BAR + 256;
    static constexpr int SMEM = OFF_ITEMS + 4 * kLocalItems + 1024;
    static constexpr int CTAS = 2 * (SMEM + 1024) <= 228 * 1024 ? 2 : 1;
    static constexpr int TM_QH = 0, TM_QL = D;      // TMEM mode only
    static constexpr int TM_S = QT ? 2 * D : 0, TM_PL = TM_S + 2 * BN, TM_O = TM_PL + BN;
    // The tensor core's accumulation into TMEM is not round-to-nearest, and a
    // row's O gathers many thousands of products: accumulated there over the
    // whole key range, an all-positive V drifts by ~1e-5 at T = 1024.  So PV
    // restarts its TMEM sum (TM_O) every kFold key tiles and the softmax
    // warpgroup adds each group into the running output in fp32 -- in TMEM
    // (TM_A) where the columns allow, else in registers (d 128).
    static constexpr bool ACC_TMEM = TM_O + 2 * D <= (QT ? 512 : (D <= 32 ? 256 : 512));
    static constexpr int TM_A = TM_O + D;
    static constexpr int TM_COLS = QT || TM_A + D > 256 ? 512 : 256;
    // per-thread registers after setmaxnreg: warpgroup 0, splitters, softmax
    // (two CTAs per SM: 384 x 80 at launch = 128 x (32 + 56 + 152); one CTA:
    // 384 x 168 at launch >= 128 x (64 + 160 + 232), or 128 x (64 + 200 + 232)
    // at d = 96).  ptxas allocates each role's code within its budget: with
    // one CTA per SM these budgets compile without spills; at d = 32 (two
    // CTAs per SM) no split of the 240 registers does, and 32/56/152 leaves
    // the fewest (80 bytes, against 136 for 40/56/144), which ran fastest.
    static constexpr int REG_MMA = CTAS == 2 ? 32 : 64;
    static constexpr int REG_SPLIT = CTAS == 2 ? 56 : (D == 96 ? 200 : 160);
    static constexpr int REG_SOFT = CTAS == 2 ? 152 : 232;
    static_assert(CTAS == 2 ? REG_MMA + REG_SPLIT + REG_SOFT <= 3 * 80 : REG_MMA + REG_SPLIT + REG_SOFT <= 3 * 168,
                  "register split exceeds the launch allocation");
    static_assert(TM_O + D <= TM_COLS && (!ACC_TMEM || TM_A + D <= TM_COLS), "TMEM budget");
    static_assert(TM_COLS * CTAS <= 512, "TMEM budget per SM");
};

enum {
    B_QF = 0, B_QS, B_QE,          // query tile landed / split / free (item's last S done)
    B_KVF = 3,                     // 2: stage landed
    B_KVS = 5,                     // 2: stage split
    B_KVE = 7,                     // 2: stage free (its S and its PV finished)
    B_SF = 9,                      // 2: S buffer ready
    B_BF = 11,                     // 2: S buffer free (the PV that read its P finished)
    B_PF = 13,                     // P written (and O rescaled)
    B_OD = 14,                     // PV finished
    B_SPL = 15,                    // splitters: raw V read (before V^T overwrites it)
    B_QC = 16,                     // TMEM mode: the staged raw query tile was read
    B_COUNT = 17
};

struct Params {
    float *o;
    float *lse;
    const float *v;                // V itself, for the first query row (see the epilogue)
    long long in_stride;
    long long out_stride;
    int T, H, B, n_qt, n_items, bn;   // bn: keys per tile
    float scale_log2;              // log2(e) / sqrt(d)
    int *err;
    int use_list;
    int packable;
    const unsigned short *sched;   // [kMaxCtas + 1] list offsets, then the item lists
};

struct Item {
    int h, b, q0, n_kv;
};

__device__ __forceinline__ void split_item(const Params &p, int i, int &b, int &h, int &qt) {
    const int hb = p.H * p.B;
    qt = p.n_qt - 1 - i / hb;
    const int r = i % hb;
    h = r % p.H;
    b = r / p.H;
}
__device__ __forceinline__ Item make_item(int b, int h, int qt, int T, int bn) {
    Item it;
    it.b = b;
    it.h = h;
    it.q0 = qt * BM;
    it.n_kv = (min(it.q0 + BM, T) + bn - 1) / bn;   // key tiles up to the diagonal
    return it;
}
__device__ __forceinline__ int item_of(const Params &p, int k) {
    if (p.use_list) {
        const int idx = (int)__ldg(p.sched + blockIdx.x) + k;
        return idx < (int)__ldg(p.sched + blockIdx.x + 1) ? (int)__ldg(p.sched + kMaxCtas + 1 + idx) : -1;
    }
    const int i = (int)blockIdx.x + k * (int)gridDim.x;
    return i < p.n_items ? i : -1;
}
__device__ __forceinline__ uint32_t pack_item(const Params &p, int id) {
    int b, h, qt;
    split_item(p, id, b, h, qt);
    return (uint32_t)b | (uint32_t)h << 12 | (uint32_t)qt << 22;
}
__device__ __forceinline__ bool next_item(const Params &p, const uint32_t *items_s, int n_local, int k, Item &it) {
    if (n_local >= 0) {
        if (k >= n_local) return false;
        const uint32_t v = items_s[k];
        it = make_item((int)(v & 0xfffu), (int)((v >> 12) & 0x3ffu), (int)(v >> 22), p.T, p.bn);
        return true;
    }
    const int id = item_of(p, k);
    if (id < 0) return false;
    int b, h, qt;
    split_item(p, id, b, h, qt);
    it = make_item(b, h, qt, p.T, p.bn);
    return true;
}

// x -> (high part in place, low part at the same offset of `lo`): n floats, 16-byte vectors
__device__ __forceinline__ void split_hi_lo(float *hi, float *lo, int n, int tid, int nthreads) {
    for (int i = tid * 4; i < n; i += nthreads * 4) {
        float4 x = *reinterpret_cast<float4 *>(hi + i);
        float4 h, l;
        h.x = __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
        h.y = __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
        h.z = __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
        h.w = __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
        l.x = x.x - h.x;
        l.y = x.y - h.y;
        l.z = x.z - h.z;
        l.w = x.w - h.w;
        *reinterpret_cast<float4 *>(hi + i) = h;
        *reinterpret_cast<float4 *>(lo + i) = l;
    }
}

__device__ __forceinline__ float f4_at(const float4 &v, int c) {
    return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
}

// PARTS = 3: every product formed as xh yh + xh yl + xl yh; PARTS = 1: xh yh
// alone, for fp32 copies of bf16 inputs (exact in tf32, so their low parts are
// zero; P's low part is dropped, ~2^-11, far inside the bf16 tolerance).
template <int D, int PARTS = 3>
__global__ void __launch_bounds__(kThreads, Cfg<D>::CTAS)
fwd_tf32_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, const __grid_constant__ Params p)
{
    pdl_begin();   // launched by launch_pdl
    using C = Cfg<D>;
    constexpr int BN = C::BN;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *sb = smem_raw + (base - raw);
    const uint32_t bar0 = base + C::OFF_BAR;
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sb + C::OFF_BAR + 192);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sb + C::OFF_BAR + 196);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    uint32_t *items_s = reinterpret_cast<uint32_t *>(sb + C::OFF_ITEMS);
    int n_local = -1;
    {
        int beg = 0, n_mine;
        if (p.use_list) {
            beg = (int)__ldg(p.sched + blockIdx.x);
            n_mine = (int)__ldg(p.sched + blockIdx.x + 1) - beg;
        } else {
            n_mine = (p.n_items - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
        }
        if (p.packable && n_mine <= kLocalItems) {
            n_local = n_mine;
            for (int i = threadIdx.x; i < n_mine; i += blockDim.x)
                items_s[i] = pack_item(p, p.use_list ? (int)__ldg(p.sched + kMaxCtas + 1 + beg + i)
                                                     : (int)blockIdx.x + i * (int)gridDim.x);
        }
    }
    if (threadIdx.x == 0) {
        mbar_init(BAR(B_QF), 1);
        mbar_init(BAR(B_QS), 128);
        mbar_init(BAR(B_QE), 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(BAR(B_KVF + i), 1);
            mbar_init(BAR(B_KVS + i), 128);
            mbar_init(BAR(B_KVE + i), 2);
            mbar_init(BAR(B_SF + i), 1);
            mbar_init(BAR(B_BF + i), 1);
        }
        mbar_init(BAR(B_PF), 128);
        mbar_init(BAR(B_OD), 1);
        mbar_init(BAR(B_SPL), 128);
        mbar_init(BAR(B_QC), 128);
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
    auto wait_w = [&](int b, int parity, int code) -> bool {       // warp-wide bounded wait
        return __all_sync(0xffffffffu, mbar_wait(BAR(b), parity & 1, abort_flag, p.err, code));
    };

    // registers: see Cfg (each setmaxnreg inside its role's branch)
    if (warp < 8) {
        if (warp < 4) regs_dec<C::REG_MMA>();
        if (warp == 0) {
            // -------------------------------------------------------- producer
            const bool leader = elect_one();
            if (leader) {
                prefetch_tmap(&tq);
                prefetch_tmap(&tk);
                prefetch_tmap(&tv);
            }
            int t = 0;                                       // key tiles issued
            bool ok = true;
            for (int k = 0; ok; k++) {
                Item it;
                if (!next_item(p, items_s, n_local, k, it)) break;
                if (k > 0 && !(ok = wait_w(C::QT ? B_QC : B_QE, k - 1, 0x401))) break;
                if (leader) {
                    mbar_arrive_expect_tx(BAR(B_QF), C::QB);
#pragma unroll
                    for (int c = 0; c < C::CH; c++)
                        tma_load_3d(base + C::OFF_QH + c * (BM * 128), &tq, BAR(B_QF), it.h * D + 32 * c, it.q0, it.b);
                }
                __syncwarp();
                for (int j = 0; j < it.n_kv; j++, t++) {
                    const int st = t & 1;
                    if (t >= 2 && !(ok = wait_w(B_KVE + st, (t >> 1) - 1, 0x402))) break;
                    if (leader) {
                        const uint32_t sbase = base + C::OFF_ST + st * C::STAGE;
                        mbar_arrive_expect_tx(BAR(B_KVF + st), 2 * C::KB);
#pragma unroll
                        for (int c = 0; c < C::CH; c++) {
                            tma_load_3d(sbase + c * (BN * 128), &tk, BAR(B_KVF + st), it.h * D + 32 * c, j * BN, it.b);
                            tma_load_3d(sbase + 2 * C::KB + c * (BN * 128), &tv, BAR(B_KVF + st), it.h * D + 32 * c,
                                        j * BN, it.b);
                        }
                    }
                    __syncwarp();
                }
            }
        } else if (warp == 1) {
            // -------------------------------------------------------- S issuer
            const bool leader = elect_one();
            constexpr uint32_t idS = idesc_tf32(BM, BN, 0, 0);     // Q, K both K-major
            int t = 0;
            bool ok = true;
            for (int k = 0; ok; k++) {
                Item it;
                if (!next_item(p, items_s, n_local, k, it)) break;
                if (!(ok = wait_w(B_QS, k, 0x411))) break;
                for (int j = 0; j < it.n_kv; j++, t++) {
                    const int st = t & 1, sbuf = t & 1;
                    if (!(ok = wait_w(B_KVS + st, t >> 1, 0x412))) break;
                    if (t >= 2 && !(ok = wait_w(B_BF + sbuf, (t >> 1) - 1, 0x413))) break;
                    tc_fence_after();
                    const uint32_t kh = base + C::OFF_ST + st * C::STAGE, kl = kh + C::KB;
                    const uint32_t d_t = tmem + C::TM_S + BN * sbuf;
                    if (leader) {
                        // K-step kk: chunk kk/4 (128-byte columns), +32 bytes within it
#pragma unroll
                        for (int part = 0; part < 3; part++) {       // hh, hl, lh
                            if (part >= PARTS) break;
                            const uint32_t qa = base + (part == 2 ? C::OFF_QL : C::OFF_QH);
                            const uint32_t qt = tmem + (part == 2 ? C::TM_QL : C::TM_QH);
                            const uint32_t kb = part == 1 ? kl : kh;
#pragma unroll
                            for (int kk = 0; kk < D / 8; kk++) {
                                const uint64_t bd = sw128_desc(kb + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024);
                                if constexpr (C::QT) {
                                    mma_tf32_ts(d_t, qt + 8 * kk, bd, idS, (part > 0 || kk > 0));
                                } else {
                                    const uint64_t ad = sw128_desc(qa + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
                                    mma_tf32_ss(d_t, ad, bd, idS, (part > 0 || kk > 0));
                                }
                            }
                        }
                        mma_commit(BAR(B_SF + sbuf));
                        mma_commit(BAR(B_KVE + st));              // (this stage's K part)
                        if (j == it.n_kv - 1) mma_commit(BAR(B_QE));
                    }
                    __syncwarp();
                }
            }
        } else if (warp == 2) {
            // -------------------------------------------------------- PV issuer
            const bool leader = elect_one();
            constexpr uint32_t idO = idesc_tf32(BM, D, 0, 0);      // P from TMEM, V^T K-major
            int t = 0;
            bool ok = true;
            for (int k = 0; ok; k++) {
                Item it;
                if (!next_item(p, items_s, n_local, k, it)) break;
                for (int j = 0; j < it.n_kv; j++, t++) {
                    const int st = t & 1, sbuf = t & 1;
                    if (!(ok = wait_w(B_KVS + st, t >> 1, 0x421))) break;
                    if (!(ok = wait_w(B_PF, t, 0x422))) break;
                    tc_fence_after();
                    const uint32_t vl = base + C::OFF_ST + st * C::STAGE + 2 * C::KB, vh = vl + C::KB;
                    const uint32_t ph = tmem + C::TM_S + BN * sbuf, pl = tmem + C::TM_PL;
                    if (leader) {
                        // V^T tile [D rows][BN keys] K-major: key chunk kk/4 (32 keys, D*128
                        // bytes apart), +32 bytes per 8-key step within it
#pragma unroll
                        for (int part = 0; part < 3; part++) {       // hh, hl, lh
                            if (part >= PARTS) break;
                            const uint32_t pa = part == 2 ? pl : ph;
                            const uint32_t vb = part == 1 ? vl : vh;
#pragma unroll
                            for (int kk = 0; kk < BN / 8; kk++) {
                                const uint64_t bd = sw128_desc(vb + (kk >> 2) * (D * 128) + (kk & 3) * 32, 16, 1024);
                                mma_tf32_ts(tmem + C::TM_O, pa + 8 * kk, bd, idO, (j % kFold > 0 || part > 0 || kk > 0));
                            }
                        }
                        mma_commit(BAR(B_OD));
                        mma_commit(BAR(B_BF + sbuf));
                        mma_commit(BAR(B_KVE + st));              // (this stage's V part)
                    }
                    __syncwarp();
                }
            }
        } else if (warp >= 4) {
            // -------------------------------------------------------- splitters
            if constexpr (C::REG_SPLIT > 168) regs_inc<C::REG_SPLIT>();   // d = 96 (launched with 168)
            else regs_dec<C::REG_SPLIT>();
            const int tid = threadIdx.x - 128;
            float *qh = reinterpret_cast<float *>(sb + C::OFF_QH), *ql = reinterpret_cast<float *>(sb + C::OFF_QL);
            int t = 0;
            bool ok = true;
            for (int k = 0; ok; k++) {
                Item it;
                if (!next_item(p, items_s, n_local, k, it)) break;
                if (!(ok = wait_w(B_QF, k, 0x431))) break;
                if constexpr (C::QT) {
                    // this warp's 32 query rows (its TMEM lane quadrant), 32 columns at a
                    // time: staged raw values -> high and low parts in TMEM
                    if (k > 0 && !(ok = wait_w(B_QE, k - 1, 0x434))) break;   // the last item's S products read Q
                    tc_fence_after();
                    const int quad = warp & 3, row = quad * 32 + lane;
                    const uint32_t lb = (uint32_t)(quad * 32) << 16;
#pragma unroll 1
                    for (int c = 0; c < C::CH; c++) {
                        uint32_t hi[32], lo[32];
                        const uint8_t *src = sb + C::OFF_QH + c * (BM * 128) + row * 128;
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const float4 x = *reinterpret_cast<const float4 *>(src + ((j ^ (row & 7)) << 4));
                            const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
                            for (int u = 0; u < 4; u++) {
                                const uint32_t h = __float_as_uint(xv[u]) & 0xFFFFE000u;
                                hi[4 * j + u] = h;
                                lo[4 * j + u] = __float_as_uint(xv[u] - __uint_as_float(h));
                            }
                        }
                        tmem_st32(tmem + lb + C::TM_QH + 32 * c, hi);
                        tmem_st32(tmem + lb + C::TM_QL + 32 * c, lo);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(BAR(B_QC));
                    mbar_arrive(BAR(B_QS));
                } else {
                    split_hi_lo(qh, ql, BM * D, tid, 128);
                    fence_async_smem();
                    mbar_arrive(BAR(B_QS));
                }
                for (int j = 0; j < it.n_kv; j++, t++) {
                    const int st = t & 1;
                    if (!(ok = wait_w(B_KVF + st, t >> 1, 0x432))) break;
                    uint8_t *s0 = sb + C::OFF_ST + st * C::STAGE;
                    split_hi_lo(reinterpret_cast<float *>(s0), reinterpret_cast<float *>(s0 + C::KB), BN * D, tid,
                                128);                                                     // K
                    // V: raw tile (TMA, 128-byte swizzle, [BN keys][32-dim chunks]) ->
                    // V^T high and low parts ([D rows][32-key chunks], same swizzle).
                    // All raw values are read before the low part overwrites them.
                    uint8_t *vraw = s0 + 2 * C::KB;
                    if constexpr ((BN * D / 16) % 128 == 0) {
                        // By 4x4 micro-blocks with 16-byte loads and stores: a 32-key x
                        // 32-dim block holds an 8x8 grid of them (key group a, dim group
                        // b), and the 8 lanes of each quarter-warp take one diagonal,
                        // b = a + p (mod 8), so under either swizzle their loads hit 8
                        // different 16-byte bank groups, and so do their stores (one
                        // element per lane, as before, put 4 lanes on each bank).
                        constexpr int MB = BN * D / 16 / 128;    // micro-blocks per thread
                        float4 vr[MB][4];
#pragma unroll
                        for (int u = 0; u < MB; u++) {
                            const int m = tid + 128 * u, blk = m >> 6, a = m & 7, b = (a + ((m & 63) >> 3)) & 7;
                            const int c32 = blk % (D / 32), k32 = blk / (D / 32);
#pragma unroll
                            for (int r = 0; r < 4; r++) {
                                const int key = 32 * k32 + 4 * a + r;
                                vr[u][r] = *reinterpret_cast<const float4 *>(vraw + c32 * (BN * 128) + key * 128 +
                                                                             ((b ^ (key & 7)) << 4));
                            }
                        }
                        mbar_arrive(BAR(B_SPL));
                        if (!(ok = wait_w(B_SPL, t, 0x433))) break;
#pragma unroll
                        for (int u = 0; u < MB; u++) {
                            const int m = tid + 128 * u, blk = m >> 6, a = m & 7, b = (a + ((m & 63) >> 3)) & 7;
                            const int c32 = blk % (D / 32), k32 = blk / (D / 32);
#pragma unroll
                            for (int c = 0; c < 4; c++) {
                                const int dim = 32 * c32 + 4 * b + c;
                                const int off = k32 * (D * 128) + dim * 128 + ((a ^ (dim & 7)) << 4);
                                const float x[4] = {f4_at(vr[u][0], c), f4_at(vr[u][1], c), f4_at(vr[u][2], c),
                                                    f4_at(vr[u][3], c)};
                                float h[4], l[4];
#pragma unroll
                                for (int r = 0; r < 4; r++) {
                                    h[r] = __uint_as_float(__float_as_uint(x[r]) & 0xFFFFE000u);
                                    l[r] = x[r] - h[r];
                                }
                                *reinterpret_cast<float4 *>(s0 + 3 * C::KB + off) = make_float4(h[0], h[1], h[2], h[3]);
                                *reinterpret_cast<float4 *>(vraw + off) = make_float4(l[0], l[1], l[2], l[3]);
                            }
                        }
                    } else {
                        constexpr int PER = BN * D / 128;
                        float vr[PER];
#pragma unroll
                        for (int i = 0; i < PER; i++) {
                            const int idx = tid + 128 * i, key = idx / D, dim = idx % D;
                            vr[i] = *reinterpret_cast<const float *>(
                                vraw + (dim >> 5) * (BN * 128) + key * 128 + ((((dim & 31) >> 2) ^ (key & 7)) << 4) +
                                (dim & 3) * 4);
                        }
                        mbar_arrive(BAR(B_SPL));
                        if (!(ok = wait_w(B_SPL, t, 0x433))) break;
#pragma unroll
                        for (int i = 0; i < PER; i++) {
                            const int idx = tid + 128 * i, key = idx / D, dim = idx % D;
                            const int off = (key >> 5) * (D * 128) + dim * 128 + ((((key & 31) >> 2) ^ (dim & 7)) << 4) +
                                            (key & 3) * 4;
                            const float h = __uint_as_float(__float_as_uint(vr[i]) & 0xFFFFE000u);
                            *reinterpret_cast<float *>(s0 + 3 * C::KB + off) = h;           // V^T high
                            *reinterpret_cast<float *>(vraw + off) = vr[i] - h;             // V^T low
                        }
                    }
                    fence_async_smem();
                    mbar_arrive(BAR(B_KVS + st));
                }
            }
        }
    } else {
        // ------------------------------------------------------------ softmax
        regs_inc<C::REG_SOFT>();
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const uint32_t tPL = tmem + lane_base + C::TM_PL, tO = tmem + lane_base + C::TM_O;
        const uint32_t tA = tmem + lane_base + C::TM_A;
        float oacc[C::ACC_TMEM ? 1 : D];            // running output in registers (d 128)
        int t = 0;
        bool ok = true;
        for (int k = 0; ok; k++) {
            Item it;
            if (!next_item(p, items_s, n_local, k, it)) break;
            const int qrow = it.q0 + row;
            float m_run = -INFINITY, l_run = 0.f;
            if constexpr (!C::ACC_TMEM) {
#pragma unroll
                for (int c = 0; c < D; c++) oacc[c] = 0.f;
            }
            for (int j = 0; j < it.n_kv; j++, t++) {
                const int sbuf = t & 1;
                const uint32_t tS = tmem + lane_base + C::TM_S + BN * sbuf;
                ok = mbar_wait(BAR(B_SF + sbuf), (t >> 1) & 1, abort_flag, p.err, 0x441);
                if (!(ok = __all_sync(0xffffffffu, ok))) break;
                tc_fence_after();
                float s[BN];
#pragma unroll
                for (int h2 = 0; h2 < BN / 32; h2++) {
                    uint32_t t0[32];
                    tmem_ld32(tS + 32 * h2, t0);
                    tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; c++) s[32 * h2 + c] = __uint_as_float(t0[c]);
                }
                const int key0 = j * BN;
                if (key0 + BN - 1 > it.q0 || key0 + BN > p.T) {   // tiles touching the diagonal or T
#pragma unroll
                    for (int c = 0; c < BN; c++)
                        if (key0 + c > qrow || key0 + c >= p.T) s[c] = -INFINITY;
                }
                float mx = -INFINITY;
#pragma unroll
                for (int c = 0; c < BN; c += 2) mx = max3(mx, s[c], s[c + 1]);
                mx *= p.scale_log2;
                float alpha = 1.f;
                const bool grow = mx > m_run + 8.f;               // also true on the first tile
                if (grow) {
                    alpha = ex2(m_run - mx);
                    m_run = mx;
                    l_run *= alpha;
                }
#pragma unroll
                for (int c = 0; c < BN; c++) {
                    s[c] = ex2(fmaf(s[c], p.scale_log2, -m_run));
                    l_run += s[c];
                }
                // the previous PV has read Pl and finished with O
                if (t > 0) ok = mbar_wait(BAR(B_OD), (t - 1) & 1, abort_flag, p.err, 0x442);
                if (!(ok = __all_sync(0xffffffffu, ok))) break;
                tc_fence_after();
#pragma unroll
                for (int h2 = 0; h2 < BN / 32; h2++) {
                    uint32_t hi[32], lo[32];
#pragma unroll
                    for (int c = 0; c < 32; c++) {
                        const float x = s[32 * h2 + c];
                        const float xh = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
                        hi[c] = __float_as_uint(xh);
                        lo[c] = __float_as_uint(x - xh);
                    }
                    tmem_st32(tS + 32 * h2, hi);
                    tmem_st32(tPL + 32 * h2, lo);
                }
                // Every kFold tiles the PV sum in TM_O is folded into the running output
                // (fp32) before the next PV restarts it: running = (running + PV sum) *
                // alpha.  In between, a grown max rescales the PV sum and the running
                // output in place (warp-uniform: a warp rescales if any row needs it).
                const bool fold = j > 0 && j % kFold == 0;
                const bool have = j > kFold;           // a running output exists
                const bool resc = !fold && j > 0 && __any_sync(0xffffffffu, grow);
                if constexpr (C::ACC_TMEM) {
                    if (fold || resc) {
#pragma unroll 1
                        for (int c0 = 0; c0 < D; c0 += 16) {
                            uint32_t pv[16], oa[16];
                            tmem_ld16(tO + c0, pv);
                            if (have) tmem_ld16(tA + c0, oa);
                            tmem_wait_ld();
#pragma unroll
                            for (int c = 0; c < 16; c++) {
                                const float o = have ? __uint_as_float(oa[c]) : 0.f, v = __uint_as_float(pv[c]);
                                oa[c] = __float_as_uint(fold ? (o + v) * alpha : o * alpha);
                                pv[c] = __float_as_uint(v * alpha);
                            }
                            if (fold || have) tmem_st16(tA + c0, oa);
                            if (resc) tmem_st16(tO + c0, pv);
                        }
                    }
                } else {
                    if (fold || resc) {
#pragma unroll
                        for (int c0 = 0; c0 < D; c0 += 16) {
                            uint32_t pv[16];
                            tmem_ld16(tO + c0, pv);
                            tmem_wait_ld();
#pragma unroll
                            for (int c = 0; c < 16; c++) {
                                const float v = __uint_as_float(pv[c]);
                                oacc[c0 + c] = (oacc[c0 + c] + (fold ? v : 0.f)) * alpha;
                                pv[c] = __float_as_uint(v * alpha);
                            }
                            if (resc) tmem_st16(tO + c0, pv);
                        }
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(BAR(B_PF));
            }
            if (!ok) break;
            // epilogue: O / l of this item (the next item's first PV waits for
            // this warpgroup's next P, written after these loads completed)
            ok = mbar_wait(BAR(B_OD), (t - 1) & 1, abort_flag, p.err, 0x443);
            if (!(ok = __all_sync(0xffffffffu, ok))) break;
            tc_fence_after();
            // The first query row attends to key 0 alone: its output is V_0
            // exactly (the products would leave a 2^-22 relative error, and a
            // backward pass turns O_0 - V_0 into a nonzero gradient where the
            // exact one is zero).
            const float inv = qrow == 0 ? 1.f : 1.f / l_run;
            float *dst = p.o + ((long long)it.b * p.T + qrow) * p.out_stride + (long long)it.h * D;
            const float *v0 = p.v + (long long)it.b * p.T * p.in_stride + (long long)it.h * D;
            const bool more = it.n_kv > kFold;     // a running output exists besides the last PV sum
            auto out16 = [&](int c0, const uint32_t (&tt)[16], const float *acc) {
                if (qrow < p.T) {
                    float o[16];
#pragma unroll
                    for (int c = 0; c < 16; c++) o[c] = qrow == 0 ? v0[c0 + c] : (acc[c] + __uint_as_float(tt[c])) * inv;
#pragma unroll
                    for (int c = 0; c < 16; c += 4)
                        *reinterpret_cast<float4 *>(dst + c0 + c) = make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
                }
            };
            if constexpr (C::ACC_TMEM) {
#pragma unroll 1
                for (int c0 = 0; c0 < D; c0 += 16) {
                    uint32_t tt[16], oa[16];
                    tmem_ld16(tO + c0, tt);
                    if (more) tmem_ld16(tA + c0, oa);
                    tmem_wait_ld();
                    float acc[16];
#pragma unroll
                    for (int c = 0; c < 16; c++) acc[c] = more ? __uint_as_float(oa[c]) : 0.f;
                    out16(c0, tt, acc);
                }
            } else {
#pragma unroll
                for (int c0 = 0; c0 < D; c0 += 16) {
                    uint32_t tt[16];
                    tmem_ld16(tO + c0, tt);
                    tmem_wait_ld();
                    out16(c0, tt, oacc + c0);
                }
            }
            tc_fence_before();
            if (qrow < p.T && p.lse)
                p.lse[((long long)it.b * p.H + it.h) * p.T + qrow] = (m_run + __log2f(l_run)) * kLn2;
        }
    }

    // ---------------------------------------------------------------- teardown
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

}  // namespace ftf
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

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn_t() {
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

// 3-D view {columns, T, B} of a (B*T, stride) fp32 activation; 32 x rows boxes
// (128 bytes wide) with the 128-byte swizzle the MMA descriptors expect.
static bool cached_map_f32(CUtensorMap *m, const void *ptr, int cols, int T, int B, long long stride, int rows) {
    struct Entry { const void *ptr; int cols, T, B, rows; long long stride; CUtensorMap map; };
    static thread_local Entry cache[12];
    static thread_local int next = 0;
    for (auto &e : cache)
        if (e.ptr == ptr && e.cols == cols && e.T == T && e.B == B && e.rows == rows && e.stride == stride) {
            *m = e.map;
            return true;
        }
    auto fn = encode_fn_t();
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
    next = (next + 1) % 12;
    return true;
}

bool fwd_tf32_sm100_supported(int D, long long in_stride, long long out_stride) {
    return (D == 32 || D == 64 || D == 96 || D == 128) && in_stride % 4 == 0 && out_stride % 4 == 0 &&
           encode_fn_t() != nullptr;
}

static void lpt_schedule_tf32(const attn::ftf::Params &p, int ctas, std::vector<unsigned short> &out) {
    using namespace attn::ftf;
    std::vector<std::vector<unsigned short>> lists(ctas);
    std::priority_queue<std::pair<long long, int>, std::vector<std::pair<long long, int>>, std::greater<>> heap;
    for (int c = 0; c < ctas; c++) heap.push({0, c});
    const int hb = p.H * p.B;
    for (int i = 0; i < p.n_items; i++) {
        const int qt = p.n_qt - 1 - i / hb;
        const long long cost = (long long)(qt + 1) * BM / p.bn + 2;      // key tiles + per-item overhead
        auto [load, c] = heap.top();
        heap.pop();
        lists[c].push_back((unsigned short)i);
        heap.push({load + cost, c});
    }
    out.assign(kMaxCtas + 1 + p.n_items, 0);
    int off = 0;
    for (int c = 0; c < ctas; c++) {
        out[c] = (unsigned short)off;
        for (unsigned short v : lists[c]) out[kMaxCtas + 1 + off++] = v;
    }
    for (int c = ctas; c <= kMaxCtas; c++) out[c] = (unsigned short)off;
}

template <int D>
static int launch_tf32_t(const void *q, const void *k, const void *v, void *o, float *lse, long long in_stride,
                         long long out_stride, int B, int H, int T, int *err, cudaStream_t s, int parts) {
    void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const attn::ftf::Params) =
        parts == 1 ? attn::ftf::fwd_tf32_kernel<D, 1> : attn::ftf::fwd_tf32_kernel<D, 3>;
    using namespace attn::ftf;
    using Cg = Cfg<D>;
    CUtensorMap mq, mk, mv;
    if (!cached_map_f32(&mq, q, H * D, T, B, in_stride, BM) || !cached_map_f32(&mk, k, H * D, T, B, in_stride, Cg::BN) ||
        !cached_map_f32(&mv, v, H * D, T, B, in_stride, Cg::BN))
        return set_error(ATTN_ERR_CUDA, "3xTF32 forward: cuTensorMapEncodeTiled failed");
    Params p;
    p.o = static_cast<float *>(o);
    p.lse = lse;
    p.v = static_cast<const float *>(v);
    p.in_stride = in_stride;
    p.out_stride = out_stride;
    p.T = T;
    p.H = H;
    p.B = B;
    p.n_qt = (T + BM - 1) / BM;
    p.n_items = p.n_qt * H * B;
    p.bn = Cg::BN;
    p.scale_log2 = attn::kLog2e / sqrtf((float)D);
    p.err = err;
    const int ctas = std::max(1, std::min(std::min(Cg::CTAS * sm_count_here(), kMaxCtas), p.n_items));
    p.use_list = p.n_items <= kMaxItems;
    p.packable = B < 4096 && H < 1024 && p.n_qt < 1024;
    p.sched = nullptr;
    if (p.use_list) {
        const long long key = (((long long)T * 4096 + H) * 65536 + B) * 512 + ctas;
        p.sched = schedule_get(100 + D, key, [&](std::vector<unsigned short> &h) { lpt_schedule_tf32(p, ctas, h); });
        p.use_list = p.sched != nullptr;            // a full cache: the list-free static schedule
    }
    const size_t smem = Cg::SMEM;
    if (!ensure_smem_attr((const void *)kern, smem))
        return set_error(ATTN_ERR_CUDA, "3xTF32 forward: cannot set shared-memory size");
    if (!ensure_carveout((const void *)kern, 100))
        return set_error(ATTN_ERR_CUDA, "3xTF32 forward: cannot set the shared-memory carveout");
    return check_pdl(launch_pdl(kern, dim3(ctas), dim3(kThreads), smem, s, mq, mk, mv, p),
                     "3xTF32 forward kernel");
}

// parts = 3 for fp32 inputs; 1 for fp32 copies of bf16 inputs (see Params::parts).
int launch_fwd_tf32_sm100(int D, const void *q, const void *k, const void *v, void *o, float *lse,
                          long long in_stride, long long out_stride, int B, int H, int T, int *err,
                          cudaStream_t s, int parts) {
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15)
        return set_error(ATTN_ERR_INVALID, "3xTF32 forward: tensors must be 16-byte aligned");
    switch (D) {
        case 32: return launch_tf32_t<32>(q, k, v, o, lse, in_stride, out_stride, B, H, T, err, s, parts);
        case 64: return launch_tf32_t<64>(q, k, v, o, lse, in_stride, out_stride, B, H, T, err, s, parts);
        case 96: return launch_tf32_t<96>(q, k, v, o, lse, in_stride, out_stride, B, H, T, err, s, parts);
        case 128: return launch_tf32_t<128>(q, k, v, o, lse, in_stride, out_stride, B, H, T, err, s, parts);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "3xTF32 forward: head_dim %d", D);
    }
}

// bf16 <-> fp32 copies of (rows x cols) activations with row strides (elements);
// cols % 4 == 0, 8-byte aligned bf16 rows and 16-byte aligned fp32 rows.
__global__ void __launch_bounds__(256)
bf16_to_f32_kernel(const __nv_bfloat16 *__restrict__ src, long long sst, float *__restrict__ dst, long long dstr,
                   long long rows, int cols)
{
    attn::pdl_begin();   // launched by launch_pdl
    const int c4 = cols / 4;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < rows * c4;
         e += (long long)gridDim.x * blockDim.x) {
        const long long r = e / c4;
        const int c = (int)(e % c4) * 4;
        *reinterpret_cast<float4 *>(dst + r * dstr + c) = attn::load4(src + r * sst + c);
    }
}
__global__ void __launch_bounds__(256)
f32_to_bf16_kernel(const float *__restrict__ src, long long sst, __nv_bfloat16 *__restrict__ dst, long long dstr,
                   long long rows, int cols)
{
    attn::pdl_begin();   // launched by launch_pdl
    const int c4 = cols / 4;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < rows * c4;
         e += (long long)gridDim.x * blockDim.x) {
        const long long r = e / c4;
        const int c = (int)(e % c4) * 4;
        attn::store4(dst + r * dstr + c, *reinterpret_cast<const float4 *>(src + r * sst + c));
    }
}

void *library_workspace(int which, size_t bytes, cudaStream_t s);

// bf16 causal forward at head dims without a bf16 tensor-core kernel (32, 96,
// 128): Q, K, V are widened to fp32 (exactly: bf16 is a subset of tf32), the
// tf32 forward runs with one product per product (xh yh; the low parts are
// zero), and O is rounded back to bf16.  The fp32 copies (4 * B*T*H*d floats)
// live in a library-owned buffer; calls that use it must not overlap on the
// GPU.  Returns ATTN_ERR_NOMEM when that buffer cannot be had (the caller then
// takes the CUDA-core kernel).
int launch_fwd_bf16_via_tf32(int D, const void *q, const void *k, const void *v, void *o, float *lse,
                             long long in_stride, long long out_stride, int B, int H, int T, int *err,
                             cudaStream_t s) {
    const long long rows = (long long)B * T, hd = (long long)H * D;
    const size_t one = ((size_t)rows * hd * 4 + 255) / 256 * 256;
    char *ws = static_cast<char *>(library_workspace(3, 4 * one, s));
    if (!ws) {
        (void)cudaGetLastError();
        return set_error(ATTN_ERR_NOMEM, "bf16 forward: no room for the fp32 copies");
    }
    float *qf = reinterpret_cast<float *>(ws), *kf = reinterpret_cast<float *>(ws + one);
    float *vf = reinterpret_cast<float *>(ws + 2 * one), *of = reinterpret_cast<float *>(ws + 3 * one);
    const long long n4 = rows * (hd / 4);
    const int grid = (int)std::min<long long>((n4 + 255) / 256, 8LL * sm_count_here());
    const void *src[3] = {q, k, v};
    float *dst[3] = {qf, kf, vf};
    int st;
    for (int i = 0; i < 3; i++)
        if ((st = check_pdl(launch_pdl(bf16_to_f32_kernel, dim3(grid), dim3(256), 0, s,
                                       static_cast<const __nv_bfloat16 *>(src[i]), in_stride, dst[i], hd, rows, (int)hd),
                            "bf16 forward: widening")))
            return st;
    if ((st = launch_fwd_tf32_sm100(D, qf, kf, vf, of, lse, hd, hd, B, H, T, err, s, 1))) return st;
    return check_pdl(launch_pdl(f32_to_bf16_kernel, dim3(grid), dim3(256), 0, s, (const float *)of, hd,
                                static_cast<__nv_bfloat16 *>(o), out_stride, rows, (int)hd),
                     "bf16 forward: rounding the output");
}

}  // namespace attn_host
