// decode_ring.cu -- KV-cached decode attention over an fp32 cache for
// mid-size calls (up to 256 sequences and 256 MB of cache, too large for the
// one-CTA-per-(sequence, head) kernel of decode_head.cu), as one persistent,
// one-pass, TMA-fed kernel (sm_100a).
//
// Semantics: cached_attention, transformer.c:203-248 -- for every head, one
// query row scores cache rows 0..len-1 with (q . k_j) / sqrt(d), softmaxes
// them and sums the value rows.
//
// Design:
//   * the concatenated rows of all sequences are split evenly over one CTA
//     per SM, so every SM streams the same number of bytes and no second
//     wave exists;
//   * whole token rows (all heads, contiguous in memory) of K and V stream
//     with cp.async.bulk into a ring of ~32 KB stages, most of the SM's share
//     requested at once; the query row travels with the first stage of each
//     piece;
//   * each stage is consumed in one pass: warp h owns head h, scores the
//     stage's rows with a transposing butterfly reduction (each lane ends up
//     owning one row's score), keeps an online softmax (running max moved
//     only when a score exceeds it by more than 2^8) and accumulates the
//     value rows;
//   * a sequence split over several CTAs is merged by the CTA that finishes
//     it last: per (sequence, head) a 64-bit ticket holds (call generation,
//     count), so tickets need no clearing between calls and the call is a
//     single launch; the merge issues its loads together.
// Every mbarrier wait is bounded; a timeout records a code in the device error
// word and raises a CTA-wide abort flag, after which the producer waits
// (bounded) for the bulk copies it has in flight before the CTA exits.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "decode_launch.cuh"
#include "sm100.cuh"

namespace attn {
namespace dr {

using namespace sm100;

constexpr int kMaxSeq = 256;          // sequences per call (tables in shared memory)
constexpr int kMaxHeads = 16;         // one consumer warp per head
constexpr int kMaxGrid = 160;         // CTAs (>= the SM count); sizes the partial slots
constexpr int kRingBytes = 210 * 1024;

struct Params {
    const float *q;                   // n_seq x HD
    const char *kbase, *vbase;        // contiguous caches (kptrs == nullptr)
    const void *const *kptrs, *const *vptrs;
    const int *lens;                  // n_seq, device; NULL = max_len for all
    float *out;                       // n_seq x HD
    float *part_o;                    // [kMaxGrid + n_seq][HD]
    float *part_ml;                   // [kMaxGrid + n_seq][H][2]
    unsigned long long *tickets;      // [n_seq * H]: (generation << 32) | count
    int *err;
    long long row_bytes_stride;       // bytes between cache rows
    long long cap;                    // rows per sequence (contiguous layout)
    long long wait_limit;             // SM cycles a bounded wait may take
    long long stall_limit;            // the test hook's wait alone (the others keep wait_limit,
                                      // so only its code reaches the error word)
    int n_seq, max_len, H, stall;     // stall != 0: test hook, see the kernel
    unsigned gen;                     // this call's ticket generation (never 0)
    float qscale;                     // log2(e) / sqrt(D)
};

// Shared-memory layout for head_dim D and R rows per stage; RB (bytes of one
// token row, H*D*4) is a runtime value, so the ring's stage count is too.
struct Layout {
    int rb, stage, stages, off_meta, off_lens, off_pre, off_kp, off_vp, off_bar, n_bar, bytes;
    __host__ __device__ Layout(int H, int D, int R) {
        rb = H * D * 4;
        stage = ((2 * R + 1) * rb + 127) / 128 * 128;   // K rows | V rows | query row
        stages = kRingBytes / stage;
        if (stages > 8) stages = 8;
        off_meta = stages * stage;                      // [stages][4] ints
        off_lens = off_meta + stages * 16;              // [kMaxSeq] ints
        off_pre = off_lens + kMaxSeq * 4;               // [kMaxSeq + 1] long long
        off_kp = off_pre + (kMaxSeq + 1) * 8;           // [kMaxSeq] pointers
        off_vp = off_kp + kMaxSeq * 8;
        off_bar = off_vp + kMaxSeq * 8;
        n_bar = 2 * stages + 1;                         // FULL, EMPTY, and the test hook's barrier
        bytes = off_bar + n_bar * 8 + 16 + 128;         // + abort flag, + alignment slack
    }
};

// Sum over the 32 lanes of v[0..R) such that lane L ends up with the total of
// row r(L) (bits of L at masks 16, 8, 4 select the row; R = 8) in v[0].
template <int R>
__device__ __forceinline__ float transpose_sum(float (&v)[R], int lane) {
#pragma unroll
    for (int n = R, m = 16; n > 1; n >>= 1, m >>= 1) {
        const bool up = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; i++) {
            const float send = up ? v[i] : v[i + n / 2];
            const float keep = up ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
    }
    float s = v[0];
#pragma unroll
    for (int m = 16 / R; m >= 1; m >>= 1)             // the lane bits below the row bits
        s += __shfl_xor_sync(0xffffffffu, s, m);
    return s;
}
// row owned by lane L after transpose_sum<R>
template <int R>
__device__ __forceinline__ int row_of_lane(int lane) {
    int r = 0;
#pragma unroll
    for (int n = R, m = 16; n > 1; n >>= 1, m >>= 1) r += (lane & m) ? n / 2 : 0;
    return r;
}
// a lane that owns row j
template <int R>
__device__ __forceinline__ int lane_of_row(int j) {
    int l = 0;
#pragma unroll
    for (int n = R, m = 16; n > 1; n >>= 1, m >>= 1) {
        if (j >= n / 2) { l |= m; j -= n / 2; }
    }
    return l;
}

// CTA that owns concatenated row x when N rows are split evenly over G CTAs
// (CTA c owns [floor(c N / G), floor((c + 1) N / G))).
__device__ __forceinline__ int cta_of(long long x, long long N, int G) {
    return (int)(((x + 1) * (long long)G - 1) / N);
}

template <int D, int R>
__global__ void __launch_bounds__((kMaxHeads + 1) * 32, 1)
decode_ring_kernel(const __grid_constant__ Params p)
{
    pdl_begin();   // launched by launch_pdl
    constexpr int DL = D / 32;                       // elements of a head per lane
    const int H = p.H;
    const Layout Lo(H, D, R);
    const int S = Lo.stages, RB = Lo.rb, HD = H * D;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 127u) & ~127u;
    uint8_t *sb = smem_raw + (base - raw);
    int *meta = reinterpret_cast<int *>(sb + Lo.off_meta);
    int *lens_s = reinterpret_cast<int *>(sb + Lo.off_lens);
    long long *pre = reinterpret_cast<long long *>(sb + Lo.off_pre);
    const char **kp_s = reinterpret_cast<const char **>(sb + Lo.off_kp);
    const char **vp_s = reinterpret_cast<const char **>(sb + Lo.off_vp);
    const uint32_t bar0 = base + Lo.off_bar;
    auto FULL = [&](int s) { return bar0 + 8u * (uint32_t)s; };
    auto EMPTY = [&](int s) { return bar0 + 8u * (uint32_t)(S + s); };
    const uint32_t STALL_BAR = bar0 + 8u * (uint32_t)(2 * S);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(sb + Lo.off_bar + Lo.n_bar * 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(FULL(s), 1);
            mbar_init(EMPTY(s), H);
        }
        mbar_init(STALL_BAR, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    // lengths (clamped; bad ones flagged) and the per-sequence slab pointers,
    // all requested in one round trip
    for (int e = threadIdx.x; e < p.n_seq; e += blockDim.x) {
        int len = p.lens ? __ldg(p.lens + e) : p.max_len;
        if (len < 1 || len > p.max_len) {
            if (blockIdx.x == 0) atomicExch(p.err, 0x100 + (len < 1 ? 1 : 2));
            len = len < 1 ? 1 : p.max_len;
        }
        lens_s[e] = len;
        if (p.kptrs) {
            kp_s[e] = static_cast<const char *>(p.kptrs[e]);
            vp_s[e] = static_cast<const char *>(p.vptrs[e]);
        } else {
            kp_s[e] = p.kbase + (long long)e * p.cap * p.row_bytes_stride;
            vp_s[e] = p.vbase + (long long)e * p.cap * p.row_bytes_stride;
        }
    }
    __syncthreads();
    if (warp == 0) {                                 // prefix sums of the lengths
        const int per = (p.n_seq + 31) / 32, e0 = lane * per, e1 = min(p.n_seq, e0 + per);
        long long sum = 0;
        for (int e = e0; e < e1; e++) sum += lens_s[e];
        long long incl = sum;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const long long y = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += y;
        }
        long long run = incl - sum;
        for (int e = e0; e < e1; e++) {
            pre[e] = run;
            run += lens_s[e];
        }
        if (lane == 31) pre[p.n_seq] = incl;
    }
    __syncthreads();
    const long long N = pre[p.n_seq];
    const int G = (int)min((long long)gridDim.x, N);
    const int c = blockIdx.x;
    if (c >= G) return;
    const long long x0 = c * N / G, x1 = (c + 1) * N / G;
    // first sequence of this CTA's range: largest e with pre[e] <= x0
    auto seq_of = [&](long long x) {
        int lo = 0, hi = p.n_seq - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (pre[mid] <= x) lo = mid; else hi = mid - 1;
        }
        return lo;
    };

    if (warp == H) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int s = 0, use = 0;
            int last_use[8];
#pragma unroll
            for (int i = 0; i < 8; i++) last_use[i] = -1;
            bool ok = true;
            auto next_slot = [&]() -> bool {
                return use < S || mbar_wait(EMPTY(s), (uint32_t)((use / S + 1) & 1), abort_flag, p.err, 0x321,
                                            p.wait_limit);
            };
            for (int e = seq_of(x0); ok && e < p.n_seq && pre[e] < x1; e++) {
                const long long r0 = max(x0 - pre[e], 0LL);
                const long long r1 = min((long long)lens_s[e], x1 - pre[e]);
                const char *kb = kp_s[e], *vb = vp_s[e];
                const bool bad = (((uintptr_t)kb | (uintptr_t)vb) & 15) != 0;
                if (bad) atomicExch(p.err, 0x320);   // misaligned cache slab: its rows are not read
                for (long long b = r0; b < r1; b += R) {
                    const int nr = (int)min((long long)R, r1 - b);
                    if (!(ok = next_slot())) break;
                    int *m = meta + 4 * s;
                    m[0] = e;
                    m[1] = bad ? 0 : nr;
                    m[2] = (b == r0 ? 1 : 0) | (b + nr == r1 ? 2 : 0) | (r0 == 0 && r1 == lens_s[e] ? 4 : 0);
                    const uint32_t st = base + s * Lo.stage;
                    if (bad) {
                        mbar_arrive(FULL(s));
                    } else {
                        const bool first = b == r0;
                        mbar_arrive_expect_tx(FULL(s), 2u * nr * RB + (first ? RB : 0));
                        if (p.row_bytes_stride == RB) {
                            bulk_load(st, kb + b * RB, nr * RB, FULL(s));
                            bulk_load(st + R * RB, vb + b * RB, nr * RB, FULL(s));
                        } else {
                            for (int i = 0; i < nr; i++) {
                                bulk_load(st + i * RB, kb + (b + i) * p.row_bytes_stride, RB, FULL(s));
                                bulk_load(st + (R + i) * RB, vb + (b + i) * p.row_bytes_stride, RB, FULL(s));
                            }
                        }
                        if (first) bulk_load(st + 2 * R * RB, p.q + (long long)e * HD, RB, FULL(s));
                        last_use[s] = use;
                    }
                    s = s + 1 == S ? 0 : s + 1;
                    use++;
                }
            }
            if (ok && next_slot()) {                 // end marker for the consumers
                meta[4 * s] = -1;
                mbar_arrive(FULL(s));
            }
            // Copies still in flight (after an abort) must land before the CTA
            // exits: wait for the last phase issued on every slot.
            if (*abort_flag) {
                volatile int no_abort = 0;
                for (int i = 0; i < S; i++)
                    if (last_use[i] >= 0)
                        mbar_wait(FULL(i), (uint32_t)((last_use[i] / S) & 1), &no_abort, nullptr, 0, 4000000000LL);
            }
        }
        __syncwarp();
        return;
    }
    if (warp >= H) return;

    // ---------------------------------------------------------------- consumers
    const int h = warp;
    const int myrow = row_of_lane<R>(lane);
    if (p.stall && h == 0) {
        // Test hook: wait on a barrier nothing arrives at, so the bounded wait
        // runs out and the abort path (error word, drained copies) runs.
        if (!mbar_wait(STALL_BAR, 0u, abort_flag, p.err, 0x32f, p.stall_limit)) return;
    }
    float qv[DL], o[DL];
    float mrun = -INFINITY, lrun = 0.f;
    int s = 0, use = 0;
    while (true) {
        if (!mbar_wait(FULL(s), (uint32_t)((use / S) & 1), abort_flag, p.err, 0x322, p.wait_limit)) break;
        const int *m = meta + 4 * s;
        const int e = m[0];
        if (e < 0) break;
        const int nr = m[1], flags = m[2];
        const float *kst = reinterpret_cast<const float *>(sb + s * Lo.stage);
        const float *vst = kst + R * (RB / 4);
        const int col = h * D + lane * DL;
        if (flags & 1) {                             // first stage of a piece: its query row, fresh state
            const float *qs = kst + 2 * R * (RB / 4);
#pragma unroll
            for (int i = 0; i < DL; i++) {
                qv[i] = qs[col + i] * p.qscale;
                o[i] = 0.f;
            }
            mrun = -INFINITY;
            lrun = 0.f;
        }
        // partial dot products of the stage's rows (rows past nr hold stale data
        // and are masked below)
        float v[R];
#pragma unroll
        for (int j = 0; j < R; j++) {
            const float *kr = kst + j * (RB / 4) + col;
            float acc = 0.f;
            if constexpr (DL == 1) {
                acc = qv[0] * kr[0];
            } else if constexpr (DL == 2) {
                const float2 k2 = *reinterpret_cast<const float2 *>(kr);
                acc = fmaf(qv[1], k2.y, qv[0] * k2.x);
            } else {
                const float4 k4 = *reinterpret_cast<const float4 *>(kr);
                acc = fmaf(qv[3], k4.w, fmaf(qv[2], k4.z, fmaf(qv[1], k4.y, qv[0] * k4.x)));
            }
            v[j] = acc;
        }
        float sc = transpose_sum<R>(v, lane);
        sc = myrow < nr ? sc : -INFINITY;
        float mx = sc;
#pragma unroll
        for (int n = R, mk = 16; n > 1; n >>= 1, mk >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, mk));
        if (mx > mrun + 8.f) {                       // also true for a piece's first stage
            const float a = ex2(mrun - mx);
            lrun *= a;
#pragma unroll
            for (int i = 0; i < DL; i++) o[i] *= a;
            mrun = mx;
        }
        const float pr = myrow < nr ? ex2(sc - mrun) : 0.f;
#pragma unroll
        for (int j = 0; j < R; j++) {
            const float pj = __shfl_sync(0xffffffffu, pr, lane_of_row<R>(j));
            if (j < nr) {
                lrun += pj;
                const float *vr = vst + j * (RB / 4) + col;
                if constexpr (DL == 1) {
                    o[0] = fmaf(pj, vr[0], o[0]);
                } else if constexpr (DL == 2) {
                    const float2 v2 = *reinterpret_cast<const float2 *>(vr);
                    o[0] = fmaf(pj, v2.x, o[0]);
                    o[1] = fmaf(pj, v2.y, o[1]);
                } else {
                    const float4 v4 = *reinterpret_cast<const float4 *>(vr);
                    o[0] = fmaf(pj, v4.x, o[0]);
                    o[1] = fmaf(pj, v4.y, o[1]);
                    o[2] = fmaf(pj, v4.z, o[2]);
                    o[3] = fmaf(pj, v4.w, o[3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(EMPTY(s));
        s = s + 1 == S ? 0 : s + 1;
        use++;
        if (!(flags & 2)) continue;
        // ---- end of a piece ---------------------------------------------------
        float *out = p.out + (long long)e * HD + col;
        if (flags & 4) {                             // the whole sequence: write the output
            const float inv = 1.f / lrun;
#pragma unroll
            for (int i = 0; i < DL; i++) out[i] = o[i] * inv;
            continue;
        }
        const long long N_ = N;
        const int c_first = cta_of(pre[e], N_, G), c_last = cta_of(pre[e + 1] - 1, N_, G);
        const long long slot = c + e;
        float *po = p.part_o + slot * HD + col;
#pragma unroll
        for (int i = 0; i < DL; i++) po[i] = o[i];
        if (lane == 0) {
            p.part_ml[(slot * H + h) * 2] = mrun;
            p.part_ml[(slot * H + h) * 2 + 1] = lrun;
        }
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            unsigned long long *t = p.tickets + (long long)e * H + h;
            unsigned long long cur = *reinterpret_cast<volatile unsigned long long *>(t);
            const unsigned long long g = (unsigned long long)p.gen << 32;
            for (int it = 0; it < (1 << 20); it++) {
                const unsigned long long want = ((cur >> 32) == p.gen) ? cur + 1 : (g | 1ull);
                const unsigned long long prev = atomicCAS(t, cur, want);
                if (prev == cur) {
                    last = (int)(want & 0xffffffffull) == c_last - c_first + 1;
                    break;
                }
                cur = prev;
            }
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence();
        // Merge this head's pieces.  Their loads go out together: the lanes
        // take 32 pieces' statistics at a time, then every lane issues 8
        // pieces' output loads before using any of them.
        const float2 *pml = reinterpret_cast<const float2 *>(p.part_ml);
        float M = -INFINITY;
        for (int c0 = c_first; c0 <= c_last; c0 += 32) {
            const int cc = c0 + lane;
            const float mv = cc <= c_last ? __ldcg(pml + (cc + e) * (long long)H + h).x : -INFINITY;
            M = fmaxf(M, mv);
        }
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
        float L = 0.f, acc[DL];
#pragma unroll
        for (int i = 0; i < DL; i++) acc[i] = 0.f;
        for (int c0 = c_first; c0 <= c_last; c0 += 32) {
            const int cc = c0 + lane;
            float2 ml = make_float2(-INFINITY, 0.f);
            if (cc <= c_last) ml = __ldcg(pml + (cc + e) * (long long)H + h);
            const float f = ml.x == -INFINITY ? 0.f : ex2(ml.x - M);
            float lf = ml.y * f;
#pragma unroll
            for (int o2 = 16; o2 > 0; o2 >>= 1) lf += __shfl_xor_sync(0xffffffffu, lf, o2);
            L += lf;
            const int n = min(32, c_last - c0 + 1);
            for (int j0 = 0; j0 < n; j0 += 8) {
                float v[8][DL];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const float *pp = p.part_o + (c0 + j0 + u + e) * (long long)HD + col;
#pragma unroll
                    for (int i = 0; i < DL; i++) v[u][i] = j0 + u < n ? __ldcg(pp + i) : 0.f;
                }
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const float fu = __shfl_sync(0xffffffffu, f, (j0 + u) & 31);
#pragma unroll
                    for (int i = 0; i < DL; i++) acc[i] = fmaf(v[u][i], fu, acc[i]);
                }
            }
        }
        const float inv = 1.f / L;
#pragma unroll
        for (int i = 0; i < DL; i++) out[i] = acc[i] * inv;
    }
}

}  // namespace dr
}  // namespace attn

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace attn_host {

bool ensure_smem_attr(const void *func, size_t bytes);

static std::atomic<unsigned> g_ring_gen{0x5bd1e995u};
static std::atomic<int> g_ring_stall{0};

// Test hook: the next `n` launches of the ring decode make one consumer wait on
// a barrier nothing arrives at, with a bound of `limit` SM cycles.
static std::atomic<long long> g_ring_stall_limit{0};
void decode_ring_force_timeout(int n, long long limit) {
    g_ring_stall_limit.store(limit);
    g_ring_stall.store(n);
}

// Calls this kernel takes: fp32 caches, one warp per head (H <= 16), head_dim
// 32/64/128, rows of at most 4 KB, few sequences, and a small total (at most
// 256 MB of K and V by the max_len bound).  Larger calls stream well through
// the split kernels, whose many CTAs cover the SMs several times over.
bool decode_ring_ok(const DecodeLaunch &L) {
    if (L.kv_dtype != ATTN_F32 || L.heads > attn::dr::kMaxHeads || L.n_seq > attn::dr::kMaxSeq) return false;
    if (L.head_dim != 32 && L.head_dim != 64 && L.head_dim != 128) return false;
    const long long rb = (long long)L.heads * L.head_dim * 4;
    if (rb > 4096 || rb % 16) return false;
    if ((L.row_stride * 4) % 16) return false;
    if (((uintptr_t)L.q & 15)) return false;
    if (!L.kptrs && (((uintptr_t)L.kbase | (uintptr_t)L.vbase) & 15)) return false;
    const long long bytes = 2LL * L.n_seq * (long long)L.max_len * rb;
    return bytes <= (256LL << 20);
}

size_t decode_ring_ws_bytes(int n_seq, int heads, int head_dim) {
    size_t r = ((size_t)n_seq * heads * 8 + 255) / 256 * 256;                                    // tickets
    r += ((size_t)(attn::dr::kMaxGrid + n_seq) * heads * 2 * sizeof(float) + 255) / 256 * 256;    // part_ml
    r += ((size_t)(attn::dr::kMaxGrid + n_seq) * heads * head_dim * sizeof(float) + 255) / 256 * 256;
    return r;
}

template <int D, int R>
static int launch_ring_t(const DecodeLaunch &L) {
    using namespace attn::dr;
    Params p;
    char *ws = static_cast<char *>(L.ws);
    const int H = L.heads;
    const size_t t_bytes = ((size_t)L.n_seq * H * 8 + 255) / 256 * 256;
    const size_t ml_bytes = ((size_t)(kMaxGrid + L.n_seq) * H * 2 * sizeof(float) + 255) / 256 * 256;
    p.tickets = reinterpret_cast<unsigned long long *>(ws);
    p.part_ml = reinterpret_cast<float *>(ws + t_bytes);
    p.part_o = reinterpret_cast<float *>(ws + t_bytes + ml_bytes);
    p.q = L.q;
    p.kbase = static_cast<const char *>(L.kbase);
    p.vbase = static_cast<const char *>(L.vbase);
    p.kptrs = L.kptrs;
    p.vptrs = L.vptrs;
    p.lens = L.lens;
    p.out = L.out;
    p.err = L.err;
    p.row_bytes_stride = L.row_stride * 4;
    p.cap = L.cap;
    p.n_seq = L.n_seq;
    p.max_len = L.max_len;
    p.H = H;
    p.qscale = attn::kLog2e / sqrtf((float)D);
    p.wait_limit = 4000000000LL;
    p.stall = 0;
    p.stall_limit = 0;
    if (g_ring_stall.load() > 0) {
        g_ring_stall.fetch_sub(1);
        p.stall = 1;
        p.stall_limit = g_ring_stall_limit.load();
    }
    unsigned g = g_ring_gen.fetch_add(1) + 1;
    if (g == 0) g = g_ring_gen.fetch_add(1) + 1;
    p.gen = g;
    const Layout Lo(H, D, R);
    const size_t smem = (size_t)Lo.bytes;
    if (Lo.stages < 3) return set_error(ATTN_ERR_UNSUPPORTED, "decode: ring stages");
    if (!ensure_smem_attr((const void *)decode_ring_kernel<D, R>, smem))
        return set_error(ATTN_ERR_CUDA, "decode: cannot set shared-memory size");
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int grid = std::max(1, std::min(std::min(sms, kMaxGrid), L.n_seq * L.max_len));
    return check_pdl(launch_pdl(decode_ring_kernel<D, R>, dim3(grid), dim3((H + 1) * 32), smem, L.stream, p),
                     "decode_ring_kernel");
}

int launch_decode_ring(const DecodeLaunch &L) {
    const int rb = L.heads * L.head_dim * 4;
    const bool r8 = rb <= 2048;
    switch (L.head_dim) {
        case 32: return r8 ? launch_ring_t<32, 8>(L) : launch_ring_t<32, 4>(L);
        case 64: return r8 ? launch_ring_t<64, 8>(L) : launch_ring_t<64, 4>(L);
        case 128: return r8 ? launch_ring_t<128, 8>(L) : launch_ring_t<128, 4>(L);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "decode: no ring kernel for head_dim %d", L.head_dim);
    }
}

}  // namespace attn_host

extern "C" ATTN_API int attn_debug_decode_timeout(int launches, long long limit_cycles) {
    if (launches < 0 || (launches > 0 && limit_cycles < 1000))
        return attn_host::set_error(ATTN_ERR_INVALID, "attn_debug_decode_timeout: launches %d, limit %lld "
                                    "(the limit must be >= 1000 cycles)", launches, limit_cycles);
    attn_host::decode_ring_force_timeout(launches, limit_cycles);
    return ATTN_OK;
}
