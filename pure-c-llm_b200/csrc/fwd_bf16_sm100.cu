// fwd_bf16_sm100.cu -- causal flash forward on the Blackwell tensor cores.
//
// Semantics: attention_forward, train.c:339-370, with bf16 Q/K/V/O and fp32
// scores, softmax statistics and accumulators (the tolerance of this path is
// stated against fp32 attention over the same bf16 inputs).
//
// Persistent kernel: one CTA per SM walks a list of work items; an item is a
// pair of consecutive 128-row query tiles of one (batch, head).  The host
// orders the items longest-first and deals them to CTAs greedily (LPT), so
// the causal triangle's uneven item costs balance across SMs.  12 warps:
//   warp 0      TMA producer: Q tiles into a double buffer (the next item's Q
//               loads while the current item runs), K_j/V_j into a 4-stage
//               ring that runs across item boundaries, K and V on separate
//               barriers (the S issuer needs only K).  The first item's Q and
//               K_0 are requested during the set-up, by the thread that
//               initialises the barriers.
//   warps 1-3   MMA issuers, tcgen05.mma kind::f16 with fp32 accumulators in
//               TMEM: warp 1 issues S_i = Q_i K_j^T for both query tiles (both
//               operands in shared memory), warp 2 O_0 += P_0 V_j and warp 3
//               O_1 += P_1 V_j (P from TMEM, V from shared memory)
//   warps 4-7   softmax for query tile 0 of each item; warps 8-11 for tile 1.
//               A thread owns one query row (= one TMEM lane): it reads its S
//               row with tcgen05.ld, keeps the running max/sum, writes its row
//               of P (bf16 pairs) back into TMEM with tcgen05.st, and rescales
//               its O row in TMEM when the max grew by more than 2^8
//               (otherwise the stale max is kept; the final normalisation uses
//               the same max for O and the sum).
// The S issuer runs one key tile ahead: it issues S_{j+1} as soon as a
// warpgroup has drained S_j, so a warpgroup never waits for its next scores,
// and the first S of the next item while the warpgroups still finish the
// current one; that item's first PV waits until the warpgroup has read out
// the previous O.
//
// Epilogue: each softmax warp stages its 32 normalised output rows in shared
// memory (bf16, 128-byte swizzle) and writes them with one TMA store, which
// also drops the rows past T.
// TMEM: S0 cols [0,128), S1 [128,256), O0 [256,256+D), O1 [256+D, 256+2D),
// P0 and P1 64 columns each after the O tiles.
// Every mbarrier wait is bounded; a timeout records a code in the device
// error word, raises a CTA-wide abort flag, and all roles fall through to the
// common teardown, which frees TMEM.
#include "common.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <functional>
#include <cudaTypedefs.h>
#include <vector>

namespace attn {
namespace fa {

using namespace sm100;

constexpr int BM = 128;           // query rows per tile (TMEM lanes)
constexpr int BN = 128;           // keys per tile
constexpr int kStages = 4;
#ifndef ATTN_FWD_POLY_PAIRS
#define ATTN_FWD_POLY_PAIRS 3
#endif
constexpr int kPolyPairs = ATTN_FWD_POLY_PAIRS;   // exponential pairs (of 8) computed by exp2_poly2
constexpr int kThreads = 384;
constexpr int kMaxCtas = 160;     // >= SM count of a B200 (148)
constexpr int kMaxItems = 6144;   // schedule carried in the kernel parameters

template <int D>
struct Cfg {
    static constexpr int Q_BYTES = BM * D * 2;      // one query tile
    static constexpr int KV_BYTES = BN * D * 2;
    static constexpr int OFF_Q = 0;                 // 2 buffers x 2 query tiles
    static constexpr int OFF_KV = 4 * Q_BYTES;
    static constexpr int STAGE_BYTES = 2 * KV_BYTES;
    static constexpr int OFF_O = OFF_KV + kStages * STAGE_BYTES;   // 2 x 128 output rows, 128-byte swizzle
    static constexpr int OFF_BAR = OFF_O + 2 * BM * D * 2;
    static constexpr int OFF_ITEMS = OFF_BAR + 256;     // kLocalItems packed items
    static constexpr int SMEM = OFF_ITEMS + 4 * 256 + 1024;
    static constexpr int TM_S0 = 0, TM_S1 = 128, TM_O0 = 256, TM_O1 = 256 + D;
    static constexpr int TM_P0 = 256 + 2 * D, TM_P1 = 256 + 2 * D + BN / 2;
    static constexpr int TM_COLS = 512;
    static_assert(TM_P1 + BN / 2 <= TM_COLS, "TMEM budget");
};

// barrier slots
enum {
    B_QF = 0,                    // 2: query buffer loaded
    B_QE = 2,                    // 2: query buffer free (its last S finished)
    B_KF = 4,                    // kStages: key tile of the stage loaded
    B_VF = 4 + kStages,          // kStages: value tile of the stage loaded
    B_KVE = 4 + 2 * kStages,     // kStages: key/value stage free
    B_SF = 4 + 3 * kStages,      // 2: S ready (per warpgroup)
    B_SE = B_SF + 2,             // 2: S drained into registers
    B_PF = B_SE + 2,             // 2: P written (and O rescaled)
    B_OD = B_PF + 2,             // 2: PV finished
    B_OF = B_OD + 2,             // 2: O read out by the epilogue
    B_COUNT = B_OF + 2
};

struct Params {
    __nv_bfloat16 *o;
    float *lse;
    long long out_stride;
    int T, H, B, n_pairs, n_items;
    float scale_log2;            // log2(e) / sqrt(d)
    int *err;
    int use_list;                // 1: per-CTA lists in `sched`; 0: round-robin over items
    int packable;                // B < 4096, H < 1024, n_pairs < 1024: items fit pack_item
    const unsigned short *sched; // [kMaxCtas + 1] list offsets, then the item lists
};

struct Item {
    int h, b, q0, n0, n1, n_kv;
    bool has_q1;
};

// item i in longest-first order: pairs from the last (most key tiles) down
__device__ __forceinline__ Item decode_item(const Params &p, int i) {
    Item it;
    const int hb = p.H * p.B;
    const int pair = p.n_pairs - 1 - i / hb;
    const int r = i % hb;
    it.h = r % p.H;
    it.b = r / p.H;
    it.q0 = pair * 2 * BM;
    it.has_q1 = (it.q0 + BM) < p.T;
    it.n0 = it.q0 / BN + 1;
    it.n1 = it.has_q1 ? it.n0 + 1 : 0;
    it.n_kv = it.has_q1 ? it.n1 : it.n0;
    return it;
}

// Query tile i of a CTA's k-th item goes to warpgroup i ^ wg_swap(k).  The
// second tile of an item has one key tile more than the first; alternating
// which warpgroup takes it balances the two warpgroups over a CTA's items
// (they run ahead of each other by up to the key/value ring's depth).
#ifndef ATTN_FWD_ALTERNATE
#define ATTN_FWD_ALTERNATE 1
#endif
__device__ __forceinline__ int wg_swap(int k) { return ATTN_FWD_ALTERNATE ? (k & 1) : 0; }

// the k-th item of this CTA, or -1
__device__ __forceinline__ int item_of(const Params &p, int k) {
    if (p.use_list) {
        const int idx = (int)__ldg(p.sched + blockIdx.x) + k;
        return idx < (int)__ldg(p.sched + blockIdx.x + 1) ? (int)__ldg(p.sched + kMaxCtas + 1 + idx) : -1;
    }
    const int i = (int)blockIdx.x + k * (int)gridDim.x;
    return i < p.n_items ? i : -1;
}

// Item fields packed into 32 bits (batch 12 bits, head 10, query pair 10).
// The CTA decodes its whole list into shared memory once, at kernel start:
// every role walks the same list, and at each item boundary a dependent
// chain of global loads and integer divisions would stall all of them.
constexpr int kLocalItems = 256;
__device__ __forceinline__ uint32_t pack_item(const Params &p, int id) {
    const int hb = p.H * p.B;
    const int pair = p.n_pairs - 1 - id / hb;
    const int r = id % hb;
    return (uint32_t)(r / p.H) | (uint32_t)(r % p.H) << 12 | (uint32_t)pair << 22;
}
__device__ __forceinline__ Item unpack_item(const Params &p, uint32_t v) {
    Item it;
    it.b = (int)(v & 0xfffu);
    it.h = (int)((v >> 12) & 0x3ffu);
    it.q0 = (int)(v >> 22) * 2 * BM;
    it.has_q1 = (it.q0 + BM) < p.T;
    it.n0 = it.q0 / BN + 1;
    it.n1 = it.has_q1 ? it.n0 + 1 : 0;
    it.n_kv = it.has_q1 ? it.n1 : it.n0;
    return it;
}
// Items of this CTA: from the shared-memory copy when it holds them all
// (n_local >= 0), otherwise decoded from global memory per item.
__device__ __forceinline__ bool next_item(const Params &p, const uint32_t *items_s, int n_local, int k, Item &it) {
    if (n_local >= 0) {
        if (k >= n_local) return false;
        it = unpack_item(p, items_s[k]);
        return true;
    }
    const int id = item_of(p, k);
    if (id < 0) return false;
    it = decode_item(p, id);
    return true;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
           const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to,
           const __grid_constant__ Params p)
{
    using C = Cfg<D>;
    static_assert(D == 64, "this kernel instance covers head_dim 64");
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *sb = smem_raw + (base - raw);
    const uint32_t sQ = base + C::OFF_Q, sKV = base + C::OFF_KV, sO = base + C::OFF_O;
    const uint32_t bar0 = base + C::OFF_BAR;
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
    static_assert(8 * B_COUNT <= 224, "barrier area");
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sb + C::OFF_BAR + 224);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sb + C::OFF_BAR + 228);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t *items_s = reinterpret_cast<uint32_t *>(sb + C::OFF_ITEMS);
    int n_local = -1;                             // -1: items decoded from global memory
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
        for (int i = 0; i < 2; i++) {
            mbar_init(BAR(B_QF + i), 1);
            mbar_init(BAR(B_QE + i), 1);
            mbar_init(BAR(B_SF + i), 1);
            mbar_init(BAR(B_SE + i), 128);
            mbar_init(BAR(B_PF + i), 128);
            mbar_init(BAR(B_OD + i), 1);
            mbar_init(BAR(B_OF + i), 128);
        }
        for (int s = 0; s < kStages; s++) {
            mbar_init(BAR(B_KF + s), 1);
            mbar_init(BAR(B_VF + s), 1);
            mbar_init(BAR(B_KVE + s), 3);
        }
        *abort_flag = 0;
        fence_mbar_init();
        // The kernel is launched as a programmatic dependent of the work before
        // it on the stream, so its CTAs may start while that work finishes:
        // nothing that work may write (Q, K, V, O, lse) is touched before this
        // wait (the other threads pass the barrier after set-up first), and the
        // next kernel may be scheduled as soon as this grid has started.
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
        asm volatile("griddepcontrol.wait;" ::: "memory");
        // Every CTA's first item is item blockIdx.x (both schedules deal the
        // first items one per CTA, longest first), so its query tiles and first
        // key tile start loading before the rest of the set-up and before the
        // schedule is read.
        const Item it = decode_item(p, (int)blockIdx.x);
        prefetch_tmap(&tq);
        prefetch_tmap(&tk);
        mbar_arrive_expect_tx(BAR(B_QF), (it.has_q1 ? 2 : 1) * C::Q_BYTES);
        tma_load_3d(sQ, &tq, BAR(B_QF), it.h * D, it.q0, it.b);
        if (it.has_q1) tma_load_3d(sQ + C::Q_BYTES, &tq, BAR(B_QF), it.h * D, it.q0 + BM, it.b);
        mbar_arrive_expect_tx(BAR(B_KF), C::KV_BYTES);
        tma_load_3d(sKV, &tk, BAR(B_KF), it.h * D, 0, it.b);
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
        // warp-wide loop like the MMA issuer; the elected lane issues the copies
        const bool leader = elect_one();
        if (leader) prefetch_tmap(&tv);
        int g = 0;                                  // key/value tiles issued so far
        bool ok = true;
        for (int k = 0; ok; k++) {
            Item it;
            if (!next_item(p, items_s, n_local, k, it)) break;
            const int qb = k & 1;
            if (k >= 2 &&
                !(ok = __all_sync(0xffffffffu, mbar_wait(BAR(B_QE + qb), ((k >> 1) + 1) & 1, abort_flag, p.err, 0x201))))
                break;
            const uint32_t qdst = sQ + qb * 2 * C::Q_BYTES;
            if (leader && k > 0) {                  // item 0's query tiles were issued at set-up
                mbar_arrive_expect_tx(BAR(B_QF + qb), (it.has_q1 ? 2 : 1) * C::Q_BYTES);
                tma_load_3d(qdst, &tq, BAR(B_QF + qb), it.h * D, it.q0, it.b);
                if (it.has_q1) tma_load_3d(qdst + C::Q_BYTES, &tq, BAR(B_QF + qb), it.h * D, it.q0 + BM, it.b);
            }
            __syncwarp();
            for (int j = 0; j < it.n_kv; j++, g++) {
                const int st = g % kStages;
                if (g >= kStages &&
                    !(ok = __all_sync(0xffffffffu, mbar_wait(BAR(B_KVE + st), ((g / kStages) + 1) & 1, abort_flag,
                                                             p.err, 0x202))))
                    break;
                if (leader) {
                    const uint32_t dst = sKV + st * C::STAGE_BYTES;
                    if (g > 0) {                        // key tile 0 was issued at set-up
                        mbar_arrive_expect_tx(BAR(B_KF + st), C::KV_BYTES);
                        tma_load_3d(dst, &tk, BAR(B_KF + st), it.h * D, j * BN, it.b);
                    }
                    mbar_arrive_expect_tx(BAR(B_VF + st), C::KV_BYTES);
                    tma_load_3d(dst + C::KV_BYTES, &tv, BAR(B_VF + st), it.h * D, j * BN, it.b);
                }
                __syncwarp();
            }
        }
    } else if (warp <= 3) {
        // ------------------------------------------------------------ MMA issuers
        // Three issuing warps, so that no single thread's instruction stream
        // paces the tensor core: warp 1 issues S_i = Q_i K_j^T for both query
        // tiles, warp 2 issues O_0 += P_0 V_j, warp 3 issues O_1 += P_1 V_j.
        // Each runs its loop on the whole warp (warp-uniform state, descriptors
        // in uniform registers); the elected lane issues the MMAs and their
        // commits, which track that lane's own MMAs.  A key/value stage is
        // free once all three have released it (KVE counts three arrivals).
        const bool leader = elect_one();
        auto wait = [&](int b, int parity, int code) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(BAR(b), parity & 1, abort_flag, p.err, code));
        };
        auto release = [&](int b, bool after_mma) {   // commit (after this lane's MMAs) or plain arrive
            if (leader) {
                if (after_mma) mma_commit(BAR(b));
                else mbar_arrive(BAR(b));
            }
            __syncwarp();
        };
        int g = 0;                 // key/value tiles consumed
        bool ok = true;
        if (warp == 1) {
            constexpr uint32_t idS = idesc_bf16(BM, BN, 0, 0);   // Q, K both K-major
            int t0 = 0, t1 = 0;    // S tiles issued per warpgroup (S-empty phases)
            for (int k = 0; ok; k++) {
                Item it;
                if (!next_item(p, items_s, n_local, k, it)) break;
                const int qb = k & 1;
                if (!(ok = wait(B_QF + qb, k >> 1, 0x213))) break;
                for (int j = 0; ok && j < it.n_kv; j++) {
                    const int st = (g + j) % kStages;
                    if (!(ok = wait(B_KF + st, (g + j) / kStages, 0x214))) break;
                    // Descriptors of consecutive K-steps differ only in the
                    // start-address field, so each step adds a constant.
                    const uint64_t kd = sw128_desc(sKV + st * C::STAGE_BYTES, 16, 1024);
                    for (int i = 0; i < 2; i++) {                 // query tile i of the item
                        if (j >= (i ? it.n1 : it.n0)) continue;
                        const int w = i ^ wg_swap(k);                 // ... goes to warpgroup w
                        const int tw = w ? t1 : t0;
                        if (tw > 0 && !(ok = wait(B_SE + w, tw - 1, 0x211 + w))) break;
                        tc_fence_after();
                        const uint64_t qd = sw128_desc(sQ + (qb * 2 + i) * C::Q_BYTES, 16, 1024);
                        const uint32_t d_t = tmem + (w ? C::TM_S1 : C::TM_S0);
                        if (leader) {
#pragma unroll
                            for (int kk = 0; kk < D / 16; kk++)   // +32 bytes along K per step
                                mma_bf16_ss(d_t, qd + 2 * kk, kd + 2 * kk, idS, kk > 0);
                            mma_commit(BAR(B_SF + w));
                        }
                        __syncwarp();
                        if (w) t1++; else t0++;
                    }
                    if (!ok) break;
                    release(B_KVE + st, true);
                    if (j == it.n_kv - 1) release(B_QE + qb, true);   // this item's last S issued
                }
                g += it.n_kv;
            }
        } else {
            const int i = warp - 2;                               // warpgroup of this issuer
            constexpr uint32_t idO = idesc_bf16(BM, D, 0, 1);    // P K-major (TMEM), V MN-major
            const uint32_t pt = tmem + (i ? C::TM_P1 : C::TM_P0);
            const uint32_t d_t = tmem + (i ? C::TM_O1 : C::TM_O0);
            int t = 0, kw = 0;     // PV tiles issued, items finished (P-full / O-free phases)
            for (int k = 0; ok; k++) {
                Item it;
                if (!next_item(p, items_s, n_local, k, it)) break;
                const int n = (i ^ wg_swap(k)) ? it.n1 : it.n0;  // key tiles of this warpgroup's query tile
                for (int j = 0; ok && j < it.n_kv; j++) {
                    const int st = (g + j) % kStages;
                    // the stage's load completing orders this release after the
                    // stage's previous use was released by all three issuers
                    if (!(ok = wait(B_VF + st, (g + j) / kStages, 0x215))) break;
                    if (j >= n) {                                 // stage not used by this query tile
                        release(B_KVE + st, false);
                        continue;
                    }
                    if (j == 0 && kw > 0 && !(ok = wait(B_OF + i, kw - 1, 0x216 + i))) break;
                    if (!(ok = wait(B_PF + i, t, 0x218 + i))) break;
                    tc_fence_after();
                    const uint64_t vd = sw128_desc(sKV + st * C::STAGE_BYTES + C::KV_BYTES, 16384, 1024);
                    if (leader) {
#pragma unroll
                        for (int kk = 0; kk < BN / 16; kk++)      // 16 keys per step: 8 packed TMEM
                            mma_bf16_ts(d_t, pt + kk * 8, vd + 128 * kk, idO, (j > 0 || kk > 0));   // columns of P
                        mma_commit(BAR(B_OD + i));
                    }
                    __syncwarp();
                    release(B_KVE + st, true);
                    t++;
                }
                if (n > 0) kw++;
                g += it.n_kv;
            }
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ softmax
        regs_inc<216>();
        const int wg = (warp - 4) >> 2;
        const int quad = warp & 3;                   // TMEM lane quadrant of this warp
        const int row = quad * 32 + lane;            // query row within the tile
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const uint32_t tS = tmem + lane_base + (wg ? C::TM_S1 : C::TM_S0);
        const uint32_t tO = tmem + lane_base + (wg ? C::TM_O1 : C::TM_O0);
        const uint32_t tP = tmem + lane_base + (wg ? C::TM_P1 : C::TM_P0);
        int t = 0;                                   // global tile index of this warpgroup
        bool ok = true;
        for (int k = 0; ok; k++) {
            Item it;
            if (!next_item(p, items_s, n_local, k, it)) break;
            const int qt = wg ^ wg_swap(k);          // this warpgroup's query tile of the item
            const int n = qt ? it.n1 : it.n0;
            if (n == 0) continue;                    // no second query tile in this item
            const int qs = it.q0 + qt * BM;
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < n; j++, t++) {
                ok = mbar_wait(BAR(B_SF + wg), t & 1, abort_flag, p.err, 0x221);
                if (!(ok = __all_sync(0xffffffffu, ok))) break;   // tcgen05.ld below is warp-collective
                tc_fence_after();
                uint32_t s[128];
#pragma unroll
                for (int q4 = 0; q4 < 4; q4++) {     // (copies keep `s` in registers)
                    uint32_t tt[32];
                    tmem_ld32(tS + 32 * q4, tt);
#pragma unroll
                    for (int c = 0; c < 32; c++) s[32 * q4 + c] = tt[c];
                }
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(BAR(B_SE + wg));         // S buffer may be overwritten now

                // row max: 8 independent chains of 3-input max
                float mp[8];
#pragma unroll
                for (int i = 0; i < 8; i++) mp[i] = -INFINITY;
                if (j == n - 1) {                    // diagonal tile: keys past the query row are masked
#pragma unroll
                    for (int c = 0; c < 128; c++)
                        if (c > row) s[c] = __float_as_uint(-INFINITY);
                }
#pragma unroll
                for (int c = 0; c < 128; c += 2)
                    mp[(c >> 1) & 7] = max3(mp[(c >> 1) & 7], __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
                float mx = max3(max3(mp[0], mp[1], mp[2]), max3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
                mx *= p.scale_log2;
                float alpha = 1.f;
                const bool grow = mx > m_run + 8.f;  // also true on the first tile
                if (grow) {
                    alpha = ex2(m_run - mx);
                    m_run = mx;
                    l_run *= alpha;
                }
                // p = 2^(s*scale - m), pairwise: packed argument and sums (two
                // lanes of work per issue slot: the softmax warps share their
                // SMSPs with the MMA-issuing thread), exp2 on MUFU; bf16 pairs
                // packed on the fly for the TMEM store
                const uint64_t scale2 = f2(p.scale_log2, p.scale_log2);
                const uint64_t negm2 = f2(-m_run, -m_run);
                uint64_t lp2[4];
#pragma unroll
                for (int i = 0; i < 4; i++) lp2[i] = 0ull;
                uint32_t pk[64];
#pragma unroll
                for (int c2 = 0; c2 < 64; c2++) {
                    const uint64_t x2 = fma2(f2(__uint_as_float(s[2 * c2]), __uint_as_float(s[2 * c2 + 1])), scale2, negm2);
                    float xl, xh;
                    f2_split(x2, xl, xh);
                    // kPolyPairs of every 8 pairs on the FMA pipe, the rest on MUFU
                    const uint64_t e2 = (c2 & 7) < kPolyPairs ? exp2_poly2(x2) : f2(ex2(xl), ex2(xh));
                    lp2[c2 & 3] = add2(lp2[c2 & 3], e2);
                    float el, eh;
                    f2_split(e2, el, eh);
                    pk[c2] = pack_bf16(el, eh);
                }
                {
                    const uint64_t l2 = add2(add2(lp2[0], lp2[1]), add2(lp2[2], lp2[3]));
                    float ll, lh;
                    f2_split(l2, ll, lh);
                    l_run += ll + lh;
                }
                // P and O belong to the previous PV (maybe of the previous item) until it completes
                if (t > 0) ok = mbar_wait(BAR(B_OD + wg), (t - 1) & 1, abort_flag, p.err, 0x222);
                if (!(ok = __all_sync(0xffffffffu, ok))) break;
                tc_fence_after();
                // P row -> TMEM as bf16 pairs (keys 2c, 2c+1 in column c): the A
                // operand of the next PV product
#pragma unroll
                for (int half = 0; half < 2; half++) {
                    uint32_t tt[32];
#pragma unroll
                    for (int c = 0; c < 32; c++) tt[c] = pk[32 * half + c];
                    tmem_st32(tP + 32 * half, tt);
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
                tmem_wait_st();                      // P (and O) stores complete before the MMA reads them
                tc_fence_before();
                mbar_arrive(BAR(B_PF + wg));
            }
            if (!ok) break;
            // epilogue: O of this item, then release the O accumulator
            ok = mbar_wait(BAR(B_OD + wg), (t - 1) & 1, abort_flag, p.err, 0x223);
            if (!(ok = __all_sync(0xffffffffu, ok))) break;
            tc_fence_after();
            uint32_t o[D];
#pragma unroll
            for (int c0 = 0; c0 < D; c0 += 32) {
                uint32_t tt[32];
                tmem_ld32(tO + c0, tt);
#pragma unroll
                for (int c = 0; c < 32; c++) o[c0 + c] = tt[c];
            }
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(BAR(B_OF + wg));             // the next item's first PV may overwrite O
            // The warp stages its 32 output rows (bf16, 128-byte swizzle: the
            // 16-byte chunk c of row r sits at chunk c ^ (r & 7)) and stores
            // them with one TMA copy, which drops the rows past T.
            {
                const float inv = 1.f / l_run;
                const uint32_t srow = sO + (uint32_t)(wg * BM + row) * 128u;
                if (lane == 0) bulk_wait_read_all();     // the previous item's copy has read the rows
                __syncwarp();
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const uint32_t a = pack_bf16(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
                    const uint32_t b = pack_bf16(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
                    const uint32_t d = pack_bf16(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
                    const uint32_t e = pack_bf16(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
                    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};"
                                 ::"r"(srow + ((uint32_t)(c ^ (row & 7)) << 4)), "r"(a), "r"(b), "r"(d), "r"(e)
                                 : "memory");
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(&to, sO + (uint32_t)(wg * BM + quad * 32) * 128u, it.h * D, qs + quad * 32, it.b);
                    bulk_commit_group();
                }
            }
            const int qrow = qs + row;
            if (qrow < p.T && p.lse)
                p.lse[((long long)it.b * p.H + it.h) * p.T + qrow] = (m_run + __log2f(l_run)) * kLn2;
        }
        if (lane == 0) bulk_wait_all();              // output copies complete before the CTA exits
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
const unsigned short *schedule_get(int kernel_tag, long long key,
                                   const std::function<void(std::vector<unsigned short> &)> &build);
int sm_count_here();
bool ensure_carveout(const void *func, int percent);

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
static bool make_map(CUtensorMap *m, const void *ptr, int cols, int T, int B, long long stride, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)T, (cuuint64_t)B};
    cuuint64_t strides[2] = {(cuuint64_t)stride * 2, (cuuint64_t)stride * 2 * T};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool fwd_bf16_sm100_supported(int D, long long in_stride, long long out_stride) {
    return D == 64 && in_stride % 8 == 0 && out_stride % 8 == 0 && encode_fn() != nullptr;
}

// Longest-processing-time-first deal of the items (already in descending
// cost order) to `ctas` CTAs; item cost = key tiles of both query tiles plus
// a fixed per-item overhead.  Output: [kMaxCtas + 1] offsets, then the lists.
static void lpt_schedule(const attn::fa::Params &p, int ctas, std::vector<unsigned short> &out) {
    using namespace attn::fa;
    std::vector<std::vector<unsigned short>> lists(ctas);
    std::vector<long long> load(ctas, 0);
    const int hb = p.H * p.B;
    for (int i = 0; i < p.n_items; i++) {
        const int pair = p.n_pairs - 1 - i / hb;
        const int q0 = pair * 2 * BM;
        const bool has_q1 = (q0 + BM) < p.T;
        const int n0 = q0 / BN + 1;
        const long long cost = n0 + (has_q1 ? n0 + 1 : 0) + 2;
        const int c = (int)(std::min_element(load.begin(), load.end()) - load.begin());
        lists[c].push_back((unsigned short)i);
        load[c] += cost;
    }
    out.assign(kMaxCtas + 1 + p.n_items, 0);
    int off = 0;
    for (int c = 0; c < ctas; c++) {
        out[c] = (unsigned short)off;
        for (unsigned short v : lists[c]) out[kMaxCtas + 1 + off++] = v;
    }
    for (int c = ctas; c <= kMaxCtas; c++) out[c] = (unsigned short)off;
}

// Tensor maps are cached per (pointer, shape): encoding one costs a driver
// call, and training / benchmark loops reuse the same buffers every step.
static bool cached_map(CUtensorMap *m, const void *ptr, int cols, int T, int B, long long stride,
                       int box_rows = 128) {
    struct Entry { const void *ptr; int cols, T, B; long long stride; int box_rows; CUtensorMap map; };
    static thread_local Entry cache[16];
    static thread_local int next = 0;
    for (auto &e : cache)
        if (e.ptr == ptr && e.cols == cols && e.T == T && e.B == B && e.stride == stride && e.box_rows == box_rows) {
            *m = e.map;
            return true;
        }
    if (!make_map(m, ptr, cols, T, B, stride, box_rows)) return false;
    cache[next] = Entry{ptr, cols, T, B, stride, box_rows, *m};
    next = (next + 1) % 16;
    return true;
}

int launch_fwd_bf16_sm100(int D, const void *q, const void *k, const void *v, void *o, float *lse,
                          long long in_stride, long long out_stride, int B, int H, int T, int *err,
                          cudaStream_t s) {
    using namespace attn::fa;
    if (D != 64) return set_error(ATTN_ERR_UNSUPPORTED, "tcgen05 forward: head_dim %d", D);
    if (((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)o) & 15)
        return set_error(ATTN_ERR_INVALID, "tcgen05 forward: tensors must be 16-byte aligned");
    CUtensorMap tq, tk, tv, to;
    if (!cached_map(&tq, q, H * D, T, B, in_stride) || !cached_map(&tk, k, H * D, T, B, in_stride) ||
        !cached_map(&tv, v, H * D, T, B, in_stride) || !cached_map(&to, o, H * D, T, B, out_stride, 32))
        return set_error(ATTN_ERR_CUDA, "tcgen05 forward: cuTensorMapEncodeTiled failed");
    // The per-CTA item lists live in an immutable per-(shape, CTA count)
    // device buffer from the library's schedule cache.
    Params p;
    p.o = static_cast<__nv_bfloat16 *>(o);
    p.lse = lse;
    p.out_stride = out_stride;
    p.T = T;
    p.H = H;
    p.B = B;
    p.n_pairs = (T + 2 * BM - 1) / (2 * BM);
    p.n_items = p.n_pairs * H * B;
    p.scale_log2 = attn::kLog2e / sqrtf((float)D);
    p.err = err;
    const int ctas = std::max(1, std::min(std::min(sm_count_here(), kMaxCtas), p.n_items));
    p.use_list = p.n_items <= kMaxItems;
    p.packable = B < 4096 && H < 1024 && p.n_pairs < 1024;
    p.sched = nullptr;
    if (p.use_list) {
        const long long key = (((long long)T * 4096 + H) * 65536 + B) * 256 + ctas;
        p.sched = schedule_get(1, key, [&](std::vector<unsigned short> &h) { lpt_schedule(p, ctas, h); });
        p.use_list = p.sched != nullptr;            // a full cache: the list-free static schedule
    }
    const size_t smem = Cfg<64>::SMEM;
    if (!ensure_smem_attr((const void *)fwd_kernel<64>, smem))
        return set_error(ATTN_ERR_CUDA, "tcgen05 forward: cannot set shared-memory size");
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fwd_kernel<64>, tq, tk, tv, to, p);
    if (e != cudaSuccess) return set_error(ATTN_ERR_CUDA, "tcgen05 forward kernel: %s", cudaGetErrorString(e));
    return ATTN_OK;
}

}  // namespace attn_host
