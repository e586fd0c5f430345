// decode_stream.cu -- KV-cached decode attention over an INT8 cache as a
// TMA-fed stream (sm_100a).
//
// Semantics: cached_attention, transformer.c:203-248 -- for every head, one
// query row scores cache rows 0..len-1 with (q . k_j) / sqrt(d), softmaxes
// them and sums the value rows.  INT8 caches hold codes plus a per-(row, head)
// fp32 scale (the absmax scheme of gemm_bench.c:225-236); attention runs over
// the dequantised values code * scale.
//
// Design (HBM-bound; a few flops per byte):
//   * persistent: one CTA per SM; work items are pieces of up to P cache rows
//     of one sequence, all heads, handed out through a global counter, so the
//     ragged lengths balance across SMs without a second wave;
//   * warp 8 is a producer: it streams each piece's whole token rows (H*D
//     elements, contiguous in memory) of K and V, plus their INT8 scales, into
//     a ring of shared-memory stages with cp.async.bulk (one copy per block of
//     rows when rows are dense); the ring runs across item boundaries, so
//     DRAM always has ~100 KB per SM requested;
//   * warps 0-7 consume: warp w takes rows w and w + 8 of every 16-row block
//     (two independent rows in flight per warp); lane l holds
//     the 16-byte pieces l + 32k (k < CPL) of a row, the lanes of one head
//     reduce its dot product with shuffles (K codes meet the query's
//     fixed-point digits in dp4a; V codes become floats through a byte
//     permute, f32x2 arithmetic), and each lane keeps an online
//     softmax state (running max, sum, weighted value sum) for its heads.
//     The running max is only moved when a score exceeds it by more than 2^8
//     (base-2 domain), so rescales are rare;
//   * at the end of a piece the 8 warps' states meet in shared memory, where
//     a merger warp (warp 9) combines them into the output (one-piece
//     sequence) or the piece's partial (max, sum, output) per head while the
//     consumers go on streaming; a small kernel that follows on the stream
//     merges the pieces of longer sequences.
// Every mbarrier wait is bounded; a timeout records a code in the device
// error word and raises a CTA-wide abort flag.
#include <algorithm>

#include "common.cuh"
#include "decode_launch.cuh"
#include "sm100.cuh"

namespace attn {
namespace ds {

using namespace sm100;

constexpr int kConsumers = 8;                       // consumer warps
constexpr int kThreads = (kConsumers + 2) * 32;     // + the producer and the merger warp
constexpr int kMaxSeq = 1024;                       // sequences per call (piece table in shared memory)

struct Params {
    const float *q;
    const char *kbase, *vbase;                      // contiguous caches (kptrs == nullptr)
    const void *const *kptrs, *const *vptrs;
    const float *ksbase, *vsbase;
    const float *const *ksptrs, *const *vsptrs;
    const int *lens;
    float *out;
    float *part_o;                                  // [n_items][HD]
    float *part_ml;                                 // [n_items][H][2]
    int *starts;                                    // [n_seq + 1] first piece of each sequence
    unsigned *counter;                              // piece counter, zero before the call
    int *err;
    long long row_bytes_stride;                     // bytes between cache rows
    long long cap;
    int n_seq, max_len, piece, n_items;             // n_items = n_seq * max pieces
    float qscale;                                   // log2(e) / sqrt(D)
};

// Geometry for head_dim D and CPL 16-byte pieces per lane per row (INT8 rows).
template <int D, int CPL>
struct Geo {
    static constexpr int RB = 512 * CPL;            // bytes of one cache row (all heads)
    static constexpr int HD = RB;                   // H * D
    static constexpr int H = HD / D;
    static constexpr int LPH = D / 16;              // lanes sharing one head within a piece
    static constexpr int RPW = 2;                   // rows per consumer warp per stage
    static constexpr int R = kConsumers * RPW;      // rows per stage
    static constexpr int SCB = R * H * 4;           // scale bytes per stage (K or V)
    static constexpr int STAGE = 2 * R * RB + 2 * SCB;
    static constexpr int STAGES = 140 * 1024 / STAGE;
    static constexpr int SLOT = HD + 2 * H;         // floats of one warp's merge slot
    static constexpr int OFF_RING = 0;
    static constexpr int OFF_SLOTS = STAGES * STAGE;
    static constexpr int OFF_META = OFF_SLOTS + 2 * kConsumers * SLOT * 4;   // [STAGES][4] ints
    static constexpr int OFF_TAB = OFF_META + STAGES * 16;                   // lens, piece starts
    static constexpr int OFF_SMETA = OFF_TAB + (2 * kMaxSeq + 1) * 4;        // slot item, sequence [2][2]
    static constexpr int OFF_BAR = (OFF_SMETA + 16 + 7) / 8 * 8;
    static constexpr int N_BAR = 2 * STAGES + 4;
    static constexpr int SMEM = OFF_BAR + N_BAR * 8 + 16 + 128;
    static_assert(LPH >= 1 && LPH <= 32 && 32 % LPH == 0, "head must cover whole lanes");
    static_assert(STAGES >= 3, "ring depth");
};

// INT8 codes become floats exactly through a byte permute into the mantissa
// of 2^23 (code + 128 after flipping the sign bit) and one subtraction; two
// codes at a time as a packed pair for the f32x2 arithmetic.
__device__ __forceinline__ uint64_t codes2(uint32_t w_flipped, int j) {
    return f2(__int_as_float(__byte_perm(w_flipped, 0x4B000000u, 0x7650u + (unsigned)j)),
              __int_as_float(__byte_perm(w_flipped, 0x4B000000u, 0x7650u + (unsigned)j + 1)));
}

// bounded wait shared by all roles of this kernel
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int *abort, int *err, int code) {
    return mbar_wait(bar, parity & 1u, abort, err, code);
}

template <int D, int CPL>
__global__ void __launch_bounds__(kThreads, 1)
decode_stream_kernel(const __grid_constant__ Params p)
{
    pdl_begin();   // launched by launch_pdl
    using G = Geo<D, CPL>;
    constexpr int H = G::H, HD = G::HD, R = G::R, S = G::STAGES, RPW = G::RPW;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 127u) & ~127u;
    uint8_t *sb = smem_raw + (base - raw);
    int *meta = reinterpret_cast<int *>(sb + G::OFF_META);          // [S][4]: item, sequence, rows, flags
    int *lens_s = reinterpret_cast<int *>(sb + G::OFF_TAB);         // [n_seq] clamped lengths
    int *start_s = lens_s + kMaxSeq;                                // [n_seq + 1] first piece of each sequence
    volatile int *smeta = reinterpret_cast<volatile int *>(sb + G::OFF_SMETA);   // [2]: item, sequence
    float *slots = reinterpret_cast<float *>(sb + G::OFF_SLOTS);    // [2][kConsumers][SLOT]
    const uint32_t bar0 = base + G::OFF_BAR;
    auto FULL = [&](int s) { return bar0 + 8u * (uint32_t)s; };
    auto EMPTY = [&](int s) { return bar0 + 8u * (uint32_t)(S + s); };
    auto SLOT_FULL = [&](int par) { return bar0 + 8u * (uint32_t)(2 * S + par); };
    auto SLOT_FREE = [&](int par) { return bar0 + 8u * (uint32_t)(2 * S + 2 + par); };
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sb + G::OFF_BAR + G::N_BAR * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(FULL(s), 1);
            mbar_init(EMPTY(s), kConsumers);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(SLOT_FULL(i), kConsumers * 32);
            mbar_init(SLOT_FREE(i), 32);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    // piece table: lengths (clamped; bad ones flagged), then their prefix sums of pieces
    for (int e = threadIdx.x; e < p.n_seq; e += kThreads) {
        int len = p.lens ? __ldg(p.lens + e) : p.max_len;
        if (len < 1 || len > p.max_len) {
            if (blockIdx.x == 0) atomicExch(p.err, 0x100 + (len < 1 ? 1 : 2));
            len = len < 1 ? 1 : p.max_len;
        }
        lens_s[e] = len;
    }
    __syncthreads();
    if (warp == 0) {
        const int per = (p.n_seq + 31) / 32, e0 = lane * per, e1 = min(p.n_seq, e0 + per);
        int sum = 0;
        for (int e = e0; e < e1; e++) sum += (lens_s[e] + p.piece - 1) / p.piece;
        int incl = sum;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        int run = incl - sum;
        for (int e = e0; e < e1; e++) {
            start_s[e] = run;
            run += (lens_s[e] + p.piece - 1) / p.piece;
        }
        if (lane == 31) start_s[p.n_seq] = incl;
    }
    __syncthreads();
    const int n_pieces = start_s[p.n_seq];
    if (blockIdx.x == 0)                            // piece table for the merge kernel
        for (int e = threadIdx.x; e <= p.n_seq; e += kThreads) p.starts[e] = start_s[e];

    if (warp == kConsumers) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int s = 0, use = 0;                      // ring slot, uses of the ring so far
            bool ok = true;
            auto next_slot = [&]() -> bool {         // wait until slot s is free
                return use < S || wait_bar(EMPTY(s), (uint32_t)(use / S + 1), abort_flag, p.err, 0x301);
            };
            int v_next = (int)atomicAdd(p.counter, 1u);
            while (ok) {
                const int v = v_next;
                if (v >= n_pieces) break;
                v_next = (int)atomicAdd(p.counter, 1u);   // used next item: its latency overlaps this one
                int lo = 0, hi = p.n_seq - 1;            // sequence e with start[e] <= v < start[e + 1]
                while (lo < hi) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (start_s[mid] <= v) lo = mid; else hi = mid - 1;
                }
                const int e = lo, pc = v - start_s[e];
                const int r0 = pc * p.piece;
                const int n = min(lens_s[e] - r0, p.piece);
                const char *kb, *vb;
                const float *ksb, *vsb;
                if (p.kptrs) {
                    kb = static_cast<const char *>(p.kptrs[e]);
                    vb = static_cast<const char *>(p.vptrs[e]);
                    ksb = p.ksptrs[e];
                    vsb = p.vsptrs[e];
                } else {
                    kb = p.kbase + (long long)e * p.cap * p.row_bytes_stride;
                    vb = p.vbase + (long long)e * p.cap * p.row_bytes_stride;
                    ksb = p.ksbase + (long long)e * p.cap * H;
                    vsb = p.vsbase + (long long)e * p.cap * H;
                }
                const bool bad = (((uintptr_t)kb | (uintptr_t)vb | (uintptr_t)ksb | (uintptr_t)vsb) & 15) != 0;
                if (bad) atomicExch(p.err, 0x310);  // misaligned cache slab: its rows are not read
                for (int b = 0; b < n; b += R) {
                    const int nr = min(R, n - b);
                    if (!(ok = next_slot())) break;
                    int *m = meta + 4 * s;
                    m[0] = v;
                    m[1] = e;
                    m[2] = bad ? 0 : nr;
                    m[3] = (b == 0 ? 1 : 0) | (b + nr == n ? 2 : 0);
                    const uint32_t st = base + G::OFF_RING + s * G::STAGE;
                    if (bad) {
                        mbar_arrive(FULL(s));
                    } else {
                        mbar_arrive_expect_tx(FULL(s), 2u * nr * G::RB + 2u * nr * H * 4);
                        const long long row = r0 + b;
                        if (p.row_bytes_stride == G::RB) {
                            bulk_load(st, kb + row * G::RB, nr * G::RB, FULL(s));
                            bulk_load(st + R * G::RB, vb + row * G::RB, nr * G::RB, FULL(s));
                        } else {
                            for (int i = 0; i < nr; i++) {
                                bulk_load(st + i * G::RB, kb + (row + i) * p.row_bytes_stride, G::RB, FULL(s));
                                bulk_load(st + (R + i) * G::RB, vb + (row + i) * p.row_bytes_stride, G::RB,
                                          FULL(s));
                            }
                        }
                        bulk_load(st + 2 * R * G::RB, ksb + row * H, nr * H * 4, FULL(s));
                        bulk_load(st + 2 * R * G::RB + G::SCB, vsb + row * H, nr * H * 4, FULL(s));
                    }
                    s = (s + 1) % S;
                    use++;
                }
            }
            if (ok && next_slot()) {                 // end marker for the consumers
                meta[4 * s] = -1;
                mbar_arrive(FULL(s));
            }
        }
        __syncwarp();
    } else if (warp == kConsumers + 1) {
        // ------------------------------------------------------------ merger
        // Combines the consumer warps' states of each finished piece into the
        // output (one-piece sequence) or the piece's partial, which the merge
        // kernel that follows on the stream combines.
        const float *sl0 = slots;
        for (int k = 0;; k++) {
            const int par = k & 1;
            if (!wait_bar(SLOT_FULL(par), (uint32_t)(k >> 1), abort_flag, p.err, 0x304)) break;
            const int v = smeta[2 * par], e = smeta[2 * par + 1];
            if (v < 0) break;
            const int npc = start_s[e + 1] - start_s[e];
            const float *sl = sl0 + par * kConsumers * G::SLOT;
            float *out = p.out + (long long)e * HD;
            for (int x = lane; x < HD; x += 32) {
                const int h = x / D;
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < kConsumers; w++) M = fmaxf(M, sl[w * G::SLOT + HD + 2 * h]);
                float L = 0.f, O = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumers; w++) {
                    const float f = ex2(sl[w * G::SLOT + HD + 2 * h] - M);   // 0 for warps without rows
                    L += sl[w * G::SLOT + HD + 2 * h + 1] * f;
                    O += sl[w * G::SLOT + x] * f;
                }
                if (npc == 1) {
                    out[x] = O / L;
                } else {
                    p.part_o[(long long)v * HD + x] = O;
                    if (x % D == 0) {
                        p.part_ml[((long long)v * H + h) * 2] = M;
                        p.part_ml[((long long)v * H + h) * 2 + 1] = L;
                    }
                }
            }
            mbar_arrive(SLOT_FREE(par));             // the consumers may refill this slot set
        }
    } else {
        // ------------------------------------------------------------ consumers
        // this lane's query pieces (base-2 domain) as packed pairs; the head of each piece
        // The query as 24-bit fixed point per 16-value piece (max|q| * 2^e < 2^22),
        // three signed byte digits per value, so K codes enter the dot products
        // as raw bytes through dp4a; the int32 sums are exact.
        uint32_t qd[CPL][3][4];
        float qe[CPL];                               // 2^-e of each piece's fixed point
        int hk[CPL];
#pragma unroll
        for (int k = 0; k < CPL; k++) hk[k] = (lane + 32 * k) / G::LPH;
        float mrun[CPL], lrun[CPL];
        uint64_t o[CPL][8];
        const uint64_t bias2 = f2(-8388736.0f, -8388736.0f);
        int s = 0, use = 0, items = 0, cur_e = -1;
        bool ok = true;
        // hands a finished piece (v >= 0) or the end marker (v < 0) to the merger
        auto publish = [&](int v, int e) -> bool {
            const int par = items & 1;
            if (items >= 2 && !wait_bar(SLOT_FREE(par), (uint32_t)((items >> 1) - 1), abort_flag, p.err, 0x305))
                return false;
            if (v >= 0) {
                float *my = slots + (par * kConsumers + warp) * G::SLOT;
#pragma unroll
                for (int k = 0; k < CPL; k++) {
#pragma unroll
                    for (int x = 0; x < 8; x++) {
                        float lo, hi;
                        f2_split(o[k][x], lo, hi);
                        my[(lane + 32 * k) * 16 + 2 * x] = lo;
                        my[(lane + 32 * k) * 16 + 2 * x + 1] = hi;
                    }
                    if ((lane + 32 * k) % G::LPH == 0) {
                        my[HD + 2 * hk[k]] = mrun[k];
                        my[HD + 2 * hk[k] + 1] = lrun[k];
                    }
                }
            }
            if (warp == 0 && lane == 0) {
                smeta[2 * par] = v;
                smeta[2 * par + 1] = e;
            }
            mbar_arrive(SLOT_FULL(par));
            items++;
            return true;
        };
        while (ok) {
            if (!(ok = wait_bar(FULL(s), (uint32_t)(use / S), abort_flag, p.err, 0x303))) break;
            const int *m = meta + 4 * s;
            const int v = m[0];
            if (v < 0) {
                ok = publish(-1, 0);
                break;
            }
            const int e = m[1], nr = m[2], flags = m[3];
            if (flags & 1) {                         // first block of a piece: fresh state
                if (e != cur_e) {
                    const float *qp = p.q + (long long)e * HD;
#pragma unroll
                    for (int k = 0; k < CPL; k++) {
                        float qf[16];
                        float mxq = 0.f;
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            qf[i] = qp[(lane + 32 * k) * 16 + i] * p.qscale;
                            mxq = fmaxf(mxq, fabsf(qf[i]));
                        }
                        // scale 2^e with max|q| * 2^e < 2^22
                        // (capped: a query below 2^-79 keeps an absolute error under 2^-101)
                        const int ex = mxq > 0.f ? min(100, 21 - (int)((__float_as_uint(mxq) >> 23) & 0xff) + 127) : 0;
                        const float up = ldexpf(1.f, ex);
                        qe[k] = ldexpf(1.f, -ex);
#pragma unroll
                        for (int wd = 0; wd < 4; wd++) {
                            uint32_t d0w = 0, d1w = 0, d2w = 0;
#pragma unroll
                            for (int j = 0; j < 4; j++) {
                                const int qi = __float2int_rn(qf[4 * wd + j] * up);
                                const int d0 = ((qi & 0xff) ^ 0x80) - 0x80;
                                const int r1 = (qi - d0) >> 8;
                                const int d1 = ((r1 & 0xff) ^ 0x80) - 0x80;
                                const int d2 = (r1 - d1) >> 8;
                                d0w |= (uint32_t)(d0 & 0xff) << (8 * j);
                                d1w |= (uint32_t)(d1 & 0xff) << (8 * j);
                                d2w |= (uint32_t)(d2 & 0xff) << (8 * j);
                            }
                            qd[k][0][wd] = d0w;
                            qd[k][1][wd] = d1w;
                            qd[k][2][wd] = d2w;
                        }
                    }
                    cur_e = e;
                }
#pragma unroll
                for (int k = 0; k < CPL; k++) {
                    mrun[k] = -INFINITY;
                    lrun[k] = 0.f;
#pragma unroll
                    for (int i = 0; i < 8; i++) o[k][i] = 0ull;
                }
            }
            // this warp's rows of the block: warp + 8j, j < RPW (blocks start at
            // multiples of R rows, so row ownership repeats every block)
            const uint8_t *st = sb + G::OFF_RING + s * G::STAGE;
            float sc[RPW][CPL];
            uint4 vraw[RPW][CPL];
#pragma unroll
            for (int j = 0; j < RPW; j++) {
                const int i = warp + kConsumers * j;
                const bool live = i < nr;
                const int ii = live ? i : 0;
                const uint4 *kr = reinterpret_cast<const uint4 *>(st + ii * G::RB);
                const uint4 *vr = reinterpret_cast<const uint4 *>(st + (R + ii) * G::RB);
                const float *ks = reinterpret_cast<const float *>(st + 2 * R * G::RB) + ii * H;
#pragma unroll
                for (int k = 0; k < CPL; k++) {
                    const uint4 kw = kr[lane + 32 * k];
                    vraw[j][k] = vr[lane + 32 * k];
                    // signed codes . fixed-point query digits (exact int32 sums)
                    const int kwv[4] = {(int)kw.x, (int)kw.y, (int)kw.z, (int)kw.w};
                    int ia[3] = {0, 0, 0};
#pragma unroll
                    for (int wd = 0; wd < 4; wd++)
#pragma unroll
                        for (int d = 0; d < 3; d++) ia[d] = __dp4a(kwv[wd], (int)qd[k][d][wd], ia[d]);
                    // |sum| < 2^22: exact float through the 1.5 * 2^23 shifter
                    const float c0 = __int_as_float(ia[0] + 0x4B400000) - 12582912.f;
                    const float c1 = __int_as_float(ia[1] + 0x4B400000) - 12582912.f;
                    const float c2 = __int_as_float(ia[2] + 0x4B400000) - 12582912.f;
                    float acc = fmaf(c2, 65536.f, fmaf(c1, 256.f, c0)) * qe[k];
#pragma unroll
                    for (int off = G::LPH / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
                    sc[j][k] = live ? acc * ks[hk[k]] : -INFINITY;
                }
            }
            const float *vsb = reinterpret_cast<const float *>(st + 2 * R * G::RB + G::SCB);
#pragma unroll
            for (int k = 0; k < CPL; k++) {
                float mx = sc[0][k];
#pragma unroll
                for (int j = 1; j < RPW; j++) mx = fmaxf(mx, sc[j][k]);
                if (mx > mrun[k] + 8.f) {            // also true for a piece's first rows
                    const float a = ex2(mrun[k] - mx);
                    lrun[k] *= a;
                    const uint64_t a2 = f2(a, a);
#pragma unroll
                    for (int x = 0; x < 8; x++) o[k][x] = fma2(o[k][x], a2, 0ull);
                    mrun[k] = mx;
                }
#pragma unroll
                for (int j = 0; j < RPW; j++) {
                    const int i = warp + kConsumers * j;
                    // rows past the block contribute nothing (their score is -inf,
                    // and so may be the running max when the warp has seen no row yet)
                    const float pr = i < nr ? ex2(sc[j][k] - mrun[k]) : 0.f;
                    lrun[k] += pr;
                    const float wgt = i < nr ? pr * vsb[i * H + hk[k]] : 0.f;
                    const uint64_t w2 = f2(wgt, wgt);
                    const uint32_t w[4] = {vraw[j][k].x ^ 0x80808080u, vraw[j][k].y ^ 0x80808080u,
                                           vraw[j][k].z ^ 0x80808080u, vraw[j][k].w ^ 0x80808080u};
#pragma unroll
                    for (int x = 0; x < 8; x++)
                        o[k][x] = fma2(w2, add2(codes2(w[x >> 1], (x & 1) * 2), bias2), o[k][x]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(EMPTY(s));
            s = (s + 1) % S;
            use++;
            if (flags & 2) ok = publish(v, e);       // end of a piece: hand the states to the merger
        }
    }
    if (*abort_flag) {   // let bulk copies already in flight land before the CTA exits
        for (int i = 0; i < 1000; i++) __nanosleep(1000);
    }
}

// Sequences of more than one piece: combine the pieces' partial (max, sum,
// output) per head.  One CTA per sequence.
template <int D, int CPL>
__global__ void __launch_bounds__(256)
decode_stream_merge(const __grid_constant__ Params p)
{
    pdl_begin();   // launched by launch_pdl
    using G = Geo<D, CPL>;
    constexpr int H = G::H, HD = G::HD;
    const int e = blockIdx.x;
    const long long v0 = p.starts[e];
    const int npc = p.starts[e + 1] - (int)v0;
    if (npc <= 1) return;                           // written by the streaming kernel
    float *out = p.out + (long long)e * HD;
    for (int x = threadIdx.x; x < HD; x += blockDim.x) {
        const int h = x / D;
        float M = -INFINITY;
        for (int q2 = 0; q2 < npc; q2++) M = fmaxf(M, p.part_ml[((v0 + q2) * H + h) * 2]);
        float L = 0.f, O = 0.f;
        for (int q2 = 0; q2 < npc; q2++) {
            const float f = ex2(p.part_ml[((v0 + q2) * H + h) * 2] - M);
            L += p.part_ml[((v0 + q2) * H + h) * 2 + 1] * f;
            O += p.part_o[(v0 + q2) * HD + x] * f;
        }
        out[x] = O / L;
    }
}

}  // namespace ds
}  // namespace attn

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace attn_host {

bool ensure_smem_attr(const void *func, size_t bytes);

// Rows per piece: enough pieces for ~4 per SM at the longest length.
static int stream_piece(int max_len, int n_seq) {
    long long c = ((long long)max_len * n_seq + 4 * 148 - 1) / (4 * 148);
    c = (c + 63) / 64 * 64;
    return (int)std::max(64LL, std::min(512LL, c));
}

// Instance key (head_dim * 10 + CPL, CPL = 16-byte pieces per lane per row)
// for an INT8 row of heads*head_dim codes, or 0 when there is no instance.
static int stream_key(int heads, int head_dim, int kv_dtype) {
    if (kv_dtype != ATTN_I8) return 0;
    const long long rb = (long long)heads * head_dim;
    if (rb % 512 || heads % 4) return 0;
    const int key = head_dim * 10 + (int)(rb / 512);
    switch (key) {
        case 641: case 642: case 1282: return key;
        default: return 0;
    }
}

bool decode_stream_ok(const DecodeLaunch &L) {
    if (!stream_key(L.heads, L.head_dim, L.kv_dtype) || L.n_seq > attn::ds::kMaxSeq) return false;
    if (L.row_stride % 16) return false;
    if (!L.kptrs && (((uintptr_t)L.kbase | (uintptr_t)L.vbase | (uintptr_t)L.ksbase | (uintptr_t)L.vsbase) & 15))
        return false;
    return true;
}

bool decode_stream_shape_ok(int heads, int head_dim, int kv_dtype) {
    return stream_key(heads, head_dim, kv_dtype) != 0;
}

size_t decode_stream_ws_bytes(int n_seq, int heads, int head_dim, int max_len) {
    const int piece = stream_piece(max_len, n_seq);
    const long long n_items = (long long)n_seq * ((max_len + piece - 1) / piece);
    size_t r = ((size_t)(n_seq + 2) * sizeof(int) + 255) / 256 * 256;              // piece table + counter
    r += ((size_t)n_items * heads * 2 * sizeof(float) + 255) / 256 * 256;         // part_ml
    r += ((size_t)n_items * heads * head_dim * sizeof(float) + 255) / 256 * 256;  // part_o
    return r;
}

template <int D, int CPL>
static int launch_stream_t(const DecodeLaunch &L) {
    using namespace attn::ds;
    using Gm = Geo<D, CPL>;
    Params p;
    p.piece = stream_piece(L.max_len, L.n_seq);
    const int max_pieces = (L.max_len + p.piece - 1) / p.piece;
    p.n_items = L.n_seq * max_pieces;
    p.n_seq = L.n_seq;
    p.max_len = L.max_len;
    char *ws = static_cast<char *>(L.ws);
    const size_t t_bytes = ((size_t)(L.n_seq + 2) * sizeof(int) + 255) / 256 * 256;
    const size_t ml_bytes = ((size_t)p.n_items * Gm::H * 2 * sizeof(float) + 255) / 256 * 256;
    p.starts = reinterpret_cast<int *>(ws);
    p.counter = reinterpret_cast<unsigned *>(p.starts + L.n_seq + 1);
    p.part_ml = reinterpret_cast<float *>(ws + t_bytes);
    p.part_o = reinterpret_cast<float *>(ws + t_bytes + ml_bytes);
    cudaError_t ce = cudaMemsetAsync(p.counter, 0, sizeof(unsigned), L.stream);
    if (ce != cudaSuccess) return set_error(ATTN_ERR_CUDA, "decode: counter clear: %s", cudaGetErrorString(ce));
    p.q = L.q;
    p.kbase = static_cast<const char *>(L.kbase);
    p.vbase = static_cast<const char *>(L.vbase);
    p.kptrs = L.kptrs; p.vptrs = L.vptrs;
    p.ksbase = L.ksbase; p.vsbase = L.vsbase; p.ksptrs = L.ksptrs; p.vsptrs = L.vsptrs;
    p.lens = L.lens; p.out = L.out; p.err = L.err;
    p.row_bytes_stride = L.row_stride;
    p.cap = L.cap;
    p.qscale = attn::kLog2e / sqrtf((float)D);
    const size_t smem = Gm::SMEM;
    if (!ensure_smem_attr((const void *)decode_stream_kernel<D, CPL>, smem))
        return set_error(ATTN_ERR_CUDA, "decode: cannot set shared-memory size");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = std::max(1, std::min(sms, p.n_items));
    int st = check_pdl(launch_pdl(decode_stream_kernel<D, CPL>, dim3(grid), dim3(kThreads), smem, L.stream, p),
                       "decode_stream_kernel");
    if (st) return st;
    return check_pdl(launch_pdl(decode_stream_merge<D, CPL>, dim3(L.n_seq), dim3(256), 0, L.stream, p),
                     "decode_stream_merge");
}

int launch_decode_stream(const DecodeLaunch &L) {
    switch (stream_key(L.heads, L.head_dim, L.kv_dtype)) {
        case 641: return launch_stream_t<64, 1>(L);
        case 642: return launch_stream_t<64, 2>(L);
        case 1282: return launch_stream_t<128, 2>(L);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "decode: no streaming kernel for this shape");
    }
}

}  // namespace attn_host
