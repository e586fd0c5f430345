// decode.cu -- KV-cached decode attention, split over cache rows (sm_100a).
//
// Semantics: cached_attention, transformer.c:203-248 -- for every head, one
// query row scores cache rows 0..len-1 with (q . k_j) / sqrt(d), softmaxes
// them and sums the value rows.  INT8 caches hold codes plus a per-(row, head)
// fp32 scale (the absmax scheme of gemm_bench.c:225-236); attention runs over
// the dequantised values code * scale.
//
// Design (HBM-bound; ~0 flops per byte):
//   * one CTA per (split, head, sequence); a split is a contiguous chunk of
//     cache rows, sized on the host so the grid covers the 148 SMs several
//     times over;
//   * fp32 rows: 8 lanes per cache row, each holding head_dim/8 elements, so
//     every warp load instruction moves four full 128-byte row segments and
//     all bytes of a sector are used; int8 rows: 4 lanes per row with 16-byte
//     loads at d = 64; several row batches are loaded before any is consumed
//     to keep 8-16 KB per CTA in flight;
//   * scores live in shared memory (base-2 domain), block max / sum reduce
//     with warp shuffles;
//   * splits of one (sequence, head) are merged by the last CTA to finish
//     (threadfence + atomic ticket; nobody waits on anybody).  The tickets
//     are cleared on the stream before each launch.
#include <algorithm>

#include "common.cuh"
#include "decode_launch.cuh"
#include "sm100.cuh"

namespace attn {

struct DecodeParams {
    const float *q;                       // n_seq x H*D
    const void *kbase, *vbase;            // contiguous caches (kptrs == nullptr)
    const void *const *kptrs;             // per-sequence slabs (device array)
    const void *const *vptrs;
    const float *ksbase, *vsbase;         // INT8 scales, contiguous layout
    const float *const *ksptrs;           // INT8 scales, per-sequence slabs
    const float *const *vsptrs;
    const int *lens;                      // n_seq, device; NULL = max_len for all
    float *out;                           // n_seq x H*D
    float *part_o;                        // [n_seq*H][max_splits][D]
    float *part_ml;                       // [n_seq*H][max_splits][2]
    unsigned *tickets;                    // [n_seq*H], zero between calls
    int *err;                             // device error word
    long long row_stride;                 // elements between cache rows
    long long cap;                        // rows per sequence (contiguous layout)
    int H, max_len, max_splits, chunk;
    float qscale;                         // log2(e) / sqrt(D)
};

constexpr int kDecThreads = 128;

// Lane geometry.  fp32 rows: 8 lanes per row, lane `sub` holds the float4
// groups {sub*4 + 32k} (every warp load moves four 128-byte row segments).
// int8 rows: 4 lanes per row, lane `sub` holds D/4 consecutive bytes (16-byte
// loads at d = 64), raw words kept packed until use.
template <int D, bool I8>
struct RowSlice {
    static constexpr int LPR = I8 ? 4 : 8;                 // lanes per row
    static constexpr int ROWS = kDecThreads / LPR;         // rows per CTA pass
    static constexpr int E = D / LPR;                      // elements per lane
    static constexpr int W = I8 ? E / 4 : E;               // registers per lane
    static constexpr int UNROLL = I8 ? 8 : 4;              // row batches in flight
    uint32_t w[W];

    __device__ __forceinline__ void load(const char *row, int sub) {
        if constexpr (!I8) {
            const float *r = reinterpret_cast<const float *>(row);
#pragma unroll
            for (int k = 0; k < E / 4; k++) {
                const uint4 x = __ldg(reinterpret_cast<const uint4 *>(r + sub * 4 + 32 * k));
                w[4 * k + 0] = x.x; w[4 * k + 1] = x.y; w[4 * k + 2] = x.z; w[4 * k + 3] = x.w;
            }
        } else if constexpr (E % 16 == 0) {
            const uint4 *r = reinterpret_cast<const uint4 *>(row + sub * E);
#pragma unroll
            for (int k = 0; k < E / 16; k++) {
                const uint4 x = __ldg(r + k);
                w[4 * k + 0] = x.x; w[4 * k + 1] = x.y; w[4 * k + 2] = x.z; w[4 * k + 3] = x.w;
            }
        } else {
            const uint2 *r = reinterpret_cast<const uint2 *>(row + sub * E);
#pragma unroll
            for (int k = 0; k < E / 8; k++) {
                const uint2 x = __ldg(r + k);
                w[2 * k + 0] = x.x; w[2 * k + 1] = x.y;
            }
        }
    }
    __device__ __forceinline__ float get(int i) const {
        if constexpr (!I8) return __uint_as_float(w[i]);
        else return (float)(int8_t)((w[i / 4] >> (8 * (i % 4))) & 0xffu);
    }
    // element index (within the head) of slot i for lane `sub`
    static __device__ __forceinline__ int index(int sub, int i) {
        if constexpr (!I8) return sub * 4 + 32 * (i / 4) + (i % 4);
        else return sub * E + i;
    }
    static __device__ __forceinline__ float row_sum(float v) {
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        return v;
    }
};

template <int D, bool I8>
__global__ void __launch_bounds__(kDecThreads)
decode_split_kernel(const DecodeParams p)
{
    pdl_begin();   // launched by launch_pdl
    using Slice = RowSlice<D, I8>;
    constexpr int E = Slice::E;
    constexpr int ROWS = Slice::ROWS;
    constexpr int UNROLL = Slice::UNROLL;
    extern __shared__ float smem[];
    float *sc = smem;                         // [chunk] scores, then weights
    float *red = smem + p.chunk;              // [ROWS * D] partial outputs
    __shared__ float wred[kDecThreads / 32];
    __shared__ int last_flag;

    const int split = blockIdx.x, h = blockIdx.y, e = blockIdx.z;
    int len = p.lens ? p.lens[e] : p.max_len;
    if (len < 1 || len > p.max_len) {
        if (split == 0 && threadIdx.x == 0) atomicExch(p.err, 0x100 + (len < 1 ? 1 : 2));
        len = len < 1 ? 1 : p.max_len;
    }
    const int nsplit = (len + p.chunk - 1) / p.chunk;
    if (split >= nsplit) return;
    const int r0 = split * p.chunk;
    const int n = min(len - r0, p.chunk);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = tid / Slice::LPR, sub = tid % Slice::LPR;

    // cache bases for this sequence (element offsets in units of the cache type)
    const char *kb, *vb;
    const float *ksb = nullptr, *vsb = nullptr;
    constexpr int esz = I8 ? 1 : 4;
    if (p.kptrs) {
        kb = static_cast<const char *>(p.kptrs[e]);
        vb = static_cast<const char *>(p.vptrs[e]);
        if constexpr (I8) { ksb = p.ksptrs[e]; vsb = p.vsptrs[e]; }
    } else {
        const long long off = (long long)e * p.cap * p.row_stride;
        kb = static_cast<const char *>(p.kbase) + off * esz;
        vb = static_cast<const char *>(p.vbase) + off * esz;
        if constexpr (I8) {
            ksb = p.ksbase + (long long)e * p.cap * p.H;
            vsb = p.vsbase + (long long)e * p.cap * p.H;
        }
    }
    const long long rstride_b = p.row_stride * esz;
    const long long head_off_b = (long long)h * D * esz;

    // query slice in registers, pre-scaled into the base-2 domain
    float qv[E];
    {
        const float *qh = p.q + (long long)e * p.H * D + h * D;
#pragma unroll
        for (int i = 0; i < E; i++) qv[i] = qh[Slice::index(sub, i)] * p.qscale;
    }

    // ---- pass 1: scores of rows r0 .. r0+n-1 ----------------------------------
    for (int base = 0; base < n; base += ROWS * UNROLL) {
        Slice ks[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int r = base + u * ROWS + grp;
            if (r < n) ks[u].load(kb + (r0 + r) * rstride_b + head_off_b, sub);
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int r = base + u * ROWS + grp;
            float acc = 0.f;
            if (r < n) {
#pragma unroll
                for (int i = 0; i < E; i++) acc = fmaf(qv[i], ks[u].get(i), acc);
            }
            acc = Slice::row_sum(acc);
            if (r < n && sub == 0) {
                if constexpr (I8) acc *= __ldg(ksb + (long long)(r0 + r) * p.H + h);
                sc[r] = acc;
            }
        }
    }
    __syncthreads();

    // ---- softmax statistics of the chunk ---------------------------------------
    float m = -INFINITY;
    for (int r = tid; r < n; r += kDecThreads) m = fmaxf(m, sc[r]);
    m = warp_max(m);
    if (lane == 0) wred[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(wred[0], wred[1]), fmaxf(wred[2], wred[3]));
    __syncthreads();
    float l = 0.f;
    for (int r = tid; r < n; r += kDecThreads) {
        const float pr = exp2f(sc[r] - m);
        l += pr;
        if constexpr (I8) sc[r] = pr * __ldg(vsb + (long long)(r0 + r) * p.H + h);
        else sc[r] = pr;
    }
    l = warp_sum(l);
    if (lane == 0) wred[warp] = l;
    __syncthreads();
    l = (wred[0] + wred[1]) + (wred[2] + wred[3]);

    // ---- pass 2: weighted sum of value rows -----------------------------------
    float o[E];
#pragma unroll
    for (int i = 0; i < E; i++) o[i] = 0.f;
    for (int base = 0; base < n; base += ROWS * UNROLL) {
        Slice vs[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int r = base + u * ROWS + grp;
            if (r < n) vs[u].load(vb + (r0 + r) * rstride_b + head_off_b, sub);
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int r = base + u * ROWS + grp;
            if (r < n) {
                const float w = sc[r];
#pragma unroll
                for (int i = 0; i < E; i++) o[i] = fmaf(w, vs[u].get(i), o[i]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < E; i++) red[grp * D + Slice::index(sub, i)] = o[i];
    __syncthreads();

    float *out = p.out + (long long)e * p.H * D + h * D;
    if (nsplit == 1) {
        const float inv = 1.f / l;
        for (int c = tid; c < D; c += kDecThreads) {
            float s = 0.f;
#pragma unroll
            for (int g = 0; g < ROWS; g++) s += red[g * D + c];
            out[c] = s * inv;
        }
        return;
    }

    // ---- publish this split's partial state, last CTA merges -----------------
    const long long eh = (long long)e * p.H + h;
    float *po = p.part_o + (eh * p.max_splits + split) * D;
    for (int c = tid; c < D; c += kDecThreads) {
        float s = 0.f;
#pragma unroll
        for (int g = 0; g < ROWS; g++) s += red[g * D + c];
        po[c] = s;
    }
    if (tid == 0) {
        p.part_ml[(eh * p.max_splits + split) * 2 + 0] = m;
        p.part_ml[(eh * p.max_splits + split) * 2 + 1] = l;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(p.tickets + eh, 1u);
        last_flag = (prev == (unsigned)(nsplit - 1));
    }
    __syncthreads();
    if (!last_flag) return;
    __threadfence();

    const float *pml = p.part_ml + eh * p.max_splits * 2;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; s++) M = fmaxf(M, __ldcg(pml + 2 * s));
    float L = 0.f;
    for (int s = 0; s < nsplit; s++) L += __ldcg(pml + 2 * s + 1) * exp2f(__ldcg(pml + 2 * s) - M);
    const float invL = 1.f / L;
    const float *pob = p.part_o + eh * p.max_splits * D;
    for (int c = tid; c < D; c += kDecThreads) {
        float acc = 0.f;
        for (int s = 0; s < nsplit; s++)
            acc += __ldcg(pob + (long long)s * D + c) * exp2f(__ldcg(pml + 2 * s) - M);
        out[c] = acc * invL;
    }
    if (tid == 0) p.tickets[eh] = 0u;   // re-arm for the next call
}

// ---------------------------------------------------------------------------
// INT8 cache, all heads per CTA.  One CTA covers a chunk of rows of one
// sequence for every head, so each warp streams whole token rows (H*D bytes,
// 16 bytes per lane per load) instead of one head's 64-byte slice per CTA;
// DRAM then sees long contiguous reads.  Lane l holds the 16-byte pieces
// l + 32k (k < CPL) of a row; the D/16 lanes of one head reduce its dot
// product with shuffles.  Codes become floats exactly through a byte permute
// into the mantissa of 2^23 and one subtraction (no conversion-pipe op).
// ---------------------------------------------------------------------------
// Bytes j, j+1 of w_flipped (= word ^ 0x80808080, so byte = code + 128) as a
// packed pair of floats 2^23 + code + 128; adding -(2^23 + 128) gives the codes.
__device__ __forceinline__ uint64_t i8_pair(uint32_t w_flipped, int j) {
    return sm100::f2(__int_as_float(__byte_perm(w_flipped, 0x4B000000u, 0x7650u + (unsigned)j)),
                     __int_as_float(__byte_perm(w_flipped, 0x4B000000u, 0x7650u + (unsigned)j + 1)));
}

constexpr int kRowWarps = 8;
constexpr int kRowUnroll = 4;

template <int D, int CPL>
__global__ void __launch_bounds__(kRowWarps * 32)
decode_rows_i8_kernel(const DecodeParams p)
{
    constexpr int DPL = D / 16;            // lanes (16-byte pieces) per head
    const int H = p.H, HD = H * D;         // == 512 * CPL
    extern __shared__ float smem[];
    float *sc = smem;                      // [H][chunk] scores, then weights
    float *red = sc + H * p.chunk;         // [kRowWarps][HD] partial outputs
    float *mst = red + kRowWarps * HD;     // [H] chunk max per head
    float *lst = mst + H;                  // [H] chunk sum per head
    __shared__ int last_flag;

    const int split = blockIdx.x, e = blockIdx.y;
    int len = p.lens ? p.lens[e] : p.max_len;
    if (len < 1 || len > p.max_len) {
        if (split == 0 && threadIdx.x == 0) atomicExch(p.err, 0x100 + (len < 1 ? 1 : 2));
        len = len < 1 ? 1 : p.max_len;
    }
    const int nsplit = (len + p.chunk - 1) / p.chunk;
    if (split >= nsplit) return;
    const int r0 = split * p.chunk;
    const int n = min(len - r0, p.chunk);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const char *kb, *vb;
    const float *ksb, *vsb;
    if (p.kptrs) {
        kb = static_cast<const char *>(p.kptrs[e]);
        vb = static_cast<const char *>(p.vptrs[e]);
        ksb = p.ksptrs[e];
        vsb = p.vsptrs[e];
    } else {
        const long long off = (long long)e * p.cap * p.row_stride;
        kb = static_cast<const char *>(p.kbase) + off;
        vb = static_cast<const char *>(p.vbase) + off;
        ksb = p.ksbase + (long long)e * p.cap * H;
        vsb = p.vsbase + (long long)e * p.cap * H;
    }

    // this lane's query pieces, pre-scaled into the base-2 domain, as packed
    // fp32 pairs (the dot products run on f32x2 arithmetic: half the issue slots)
    uint64_t qv[CPL][8];
#pragma unroll
    for (int k = 0; k < CPL; k++) {
        const float *qp = p.q + (long long)e * HD + (lane + 32 * k) * 16;
#pragma unroll
        for (int i = 0; i < 8; i++) qv[k][i] = sm100::f2(qp[2 * i] * p.qscale, qp[2 * i + 1] * p.qscale);
    }
    const uint64_t bias2 = sm100::f2(-8388736.0f, -8388736.0f);

    // ---- scores: sc[h][r] = kscale * (q_h . code_h) ----------------------------
    int hk[CPL];                           // head of each of this lane's pieces
#pragma unroll
    for (int k = 0; k < CPL; k++) hk[k] = ((lane + 32 * k) * 16) / D;
    for (int base = warp; base < n; base += kRowWarps * kRowUnroll) {
        uint4 raw[kRowUnroll][CPL];
        float ksc[kRowUnroll][CPL];        // scales load together with the rows
#pragma unroll
        for (int u = 0; u < kRowUnroll; u++) {
            const int r = base + u * kRowWarps;
            if (r < n) {
                const uint4 *rowp = reinterpret_cast<const uint4 *>(kb + (long long)(r0 + r) * p.row_stride);
#pragma unroll
                for (int k = 0; k < CPL; k++) {
                    raw[u][k] = __ldg(rowp + lane + 32 * k);
                    ksc[u][k] = __ldg(ksb + (long long)(r0 + r) * H + hk[k]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kRowUnroll; u++) {
            const int r = base + u * kRowWarps;
#pragma unroll
            for (int k = 0; k < CPL; k++) {
                float acc = 0.f;
                if (r < n) {
                    const uint32_t w[4] = {raw[u][k].x ^ 0x80808080u, raw[u][k].y ^ 0x80808080u,
                                           raw[u][k].z ^ 0x80808080u, raw[u][k].w ^ 0x80808080u};
                    uint64_t a2 = 0ull;
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const uint64_t x2 = sm100::add2(i8_pair(w[i >> 1], (i & 1) * 2), bias2);
                        a2 = sm100::fma2(qv[k][i], x2, a2);
                    }
                    float al, ah;
                    sm100::f2_split(a2, al, ah);
                    acc = al + ah;
                }
#pragma unroll
                for (int o = DPL / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                if (r < n && (lane % DPL) == 0) sc[hk[k] * p.chunk + r] = acc * ksc[u][k];
            }
        }
    }
    __syncthreads();

    // ---- per-head softmax statistics of the chunk ------------------------------
    for (int h = warp; h < H; h += kRowWarps) {
        float *row = sc + h * p.chunk;
        float m = -INFINITY;
        for (int r = lane; r < n; r += 32) m = fmaxf(m, row[r]);
        m = warp_max(m);
        float l = 0.f;
        for (int r = lane; r < n; r += 32) {
            const float pr = exp2f(row[r] - m);
            l += pr;
            row[r] = pr;
        }
        l = warp_sum(l);
        if (lane == 0) { mst[h] = m; lst[h] = l; }
    }
    __syncthreads();

    // ---- weighted value rows ------------------------------------------------
    uint64_t o[CPL][8];
#pragma unroll
    for (int k = 0; k < CPL; k++)
#pragma unroll
        for (int i = 0; i < 8; i++) o[k][i] = 0ull;
    for (int base = warp; base < n; base += kRowWarps * kRowUnroll) {
        uint4 raw[kRowUnroll][CPL];
        float vsc[kRowUnroll][CPL];
#pragma unroll
        for (int u = 0; u < kRowUnroll; u++) {
            const int r = base + u * kRowWarps;
            if (r < n) {
                const uint4 *rowp = reinterpret_cast<const uint4 *>(vb + (long long)(r0 + r) * p.row_stride);
#pragma unroll
                for (int k = 0; k < CPL; k++) {
                    raw[u][k] = __ldg(rowp + lane + 32 * k);
                    vsc[u][k] = __ldg(vsb + (long long)(r0 + r) * H + hk[k]);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kRowUnroll; u++) {
            const int r = base + u * kRowWarps;
            if (r < n) {
#pragma unroll
                for (int k = 0; k < CPL; k++) {
                    const float wgt = sc[hk[k] * p.chunk + r] * vsc[u][k];
                    const uint64_t w2 = sm100::f2(wgt, wgt);
                    const uint32_t w[4] = {raw[u][k].x ^ 0x80808080u, raw[u][k].y ^ 0x80808080u,
                                           raw[u][k].z ^ 0x80808080u, raw[u][k].w ^ 0x80808080u};
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        o[k][i] = sm100::fma2(w2, sm100::add2(i8_pair(w[i >> 1], (i & 1) * 2), bias2), o[k][i]);
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < CPL; k++)
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float lo, hi;
            sm100::f2_split(o[k][i], lo, hi);
            red[warp * HD + (lane + 32 * k) * 16 + 2 * i] = lo;
            red[warp * HD + (lane + 32 * k) * 16 + 2 * i + 1] = hi;
        }
    __syncthreads();

    float *out = p.out + (long long)e * HD;
    if (nsplit == 1) {
        for (int x = threadIdx.x; x < HD; x += kRowWarps * 32) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kRowWarps; w++) s += red[w * HD + x];
            out[x] = s / lst[x / D];
        }
        return;
    }
    // ---- partial state of this split; the last split's CTA merges -----------
    float *po = p.part_o + ((long long)e * p.max_splits + split) * HD;
    for (int x = threadIdx.x; x < HD; x += kRowWarps * 32) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kRowWarps; w++) s += red[w * HD + x];
        po[x] = s;
    }
    for (int h = threadIdx.x; h < H; h += kRowWarps * 32) {
        float *pm = p.part_ml + (((long long)e * p.max_splits + split) * H + h) * 2;
        pm[0] = mst[h];
        pm[1] = lst[h];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_flag = (atomicAdd(p.tickets + e, 1u) == (unsigned)(nsplit - 1));
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    // per (split, head) rescale factors into the score area (no longer needed)
    float *fac = sc;                       // [nsplit][H], then [H] 1/L
    float *invl = sc + nsplit * H;
    for (int h = threadIdx.x; h < H; h += kRowWarps * 32) {
        float M = -INFINITY;
        for (int s = 0; s < nsplit; s++)
            M = fmaxf(M, __ldcg(p.part_ml + (((long long)e * p.max_splits + s) * H + h) * 2));
        float L = 0.f;
        for (int s = 0; s < nsplit; s++) {
            const float *pm = p.part_ml + (((long long)e * p.max_splits + s) * H + h) * 2;
            const float f = exp2f(__ldcg(pm) - M);
            fac[s * H + h] = f;
            L += __ldcg(pm + 1) * f;
        }
        invl[h] = 1.f / L;
    }
    __syncthreads();
    for (int x = threadIdx.x; x < HD; x += kRowWarps * 32) {
        const int h = x / D;
        float acc = 0.f;
        for (int s = 0; s < nsplit; s++)
            acc += __ldcg(p.part_o + ((long long)e * p.max_splits + s) * HD + x) * fac[s * H + h];
        out[x] = acc * invl[h];
    }
    if (threadIdx.x == 0) p.tickets[e] = 0u;
}

}  // namespace attn

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace attn_host {

// Rows per split: enough CTAs to cover the SMs ~8 times, 64-row granularity.
int decode_chunk(int max_len, long long units) {
    long long target = 148LL * 8;
    long long c = ((long long)max_len * units + target - 1) / target;
    c = (c + 63) / 64 * 64;
    if (c < 64) c = 64;
    if (c > 1024) c = 1024;
    return (int)c;
}

// INT8 caches whose rows are 512, 1024 or 2048 bytes take the all-heads rows
// kernel; its rows per split target ~3 CTAs per SM.
static bool rows_i8_ok(int heads, int head_dim, int kv_dtype) {
    const int hd = heads * head_dim;
    return kv_dtype == ATTN_I8 && (head_dim == 32 || head_dim == 64 || head_dim == 128) &&
           (hd == 512 || hd == 1024 || hd == 2048);
}
int rows_chunk(int max_len, int n_seq) {
    long long c = ((long long)max_len * n_seq + 443) / 444;
    c = (c + 63) / 64 * 64;
    return (int)std::max(128LL, std::min(512LL, c));
}

size_t decode_stream_ws_bytes(int n_seq, int heads, int head_dim, int max_len);
bool decode_stream_shape_ok(int heads, int head_dim, int kv_dtype);
size_t decode_i8mma_ws_bytes(int n_seq, int heads, int head_dim, int max_len);
bool decode_i8mma_shape_ok(int heads, int head_dim, int kv_dtype);
size_t decode_ring_ws_bytes(int n_seq, int heads, int head_dim);

static size_t decode_split_ws_bytes(int n_seq, int heads, int head_dim, int max_len, int kv_dtype) {
    if (rows_i8_ok(heads, head_dim, kv_dtype)) {
        const int rc = rows_chunk(max_len, n_seq);
        const long long rsplits = (max_len + rc - 1) / rc;
        size_t r = (size_t)n_seq * sizeof(unsigned);
        r = (r + 255) / 256 * 256;
        r += (size_t)n_seq * rsplits * heads * 2 * sizeof(float);
        r = (r + 255) / 256 * 256;
        r += (size_t)n_seq * rsplits * heads * head_dim * sizeof(float);
        return (r + 255) / 256 * 256;
    }
    const int chunk = decode_chunk(max_len, (long long)n_seq * heads);
    const long long splits = (max_len + chunk - 1) / chunk;
    const long long eh = (long long)n_seq * heads;
    size_t b = (size_t)eh * sizeof(unsigned);              // tickets
    b = (b + 255) / 256 * 256;
    b += (size_t)eh * splits * 2 * sizeof(float);          // part_ml
    b = (b + 255) / 256 * 256;
    b += (size_t)eh * splits * head_dim * sizeof(float);   // part_o
    return (b + 255) / 256 * 256;
}

// Covers whichever kernel the call's pointers select: the tensor-core INT8
// kernel or the streaming kernel (shape and alignment permitting), or the
// split kernels.
size_t decode_workspace_bytes(int n_seq, int heads, int head_dim, int max_len, int kv_dtype) {
    size_t b = decode_split_ws_bytes(n_seq, heads, head_dim, max_len, kv_dtype);
    if (kv_dtype == ATTN_F32) b = std::max(b, decode_ring_ws_bytes(n_seq, heads, head_dim));
    if (decode_stream_shape_ok(heads, head_dim, kv_dtype))
        b = std::max(b, decode_stream_ws_bytes(n_seq, heads, head_dim, max_len));
    if (decode_i8mma_shape_ok(heads, head_dim, kv_dtype))
        b = std::max(b, decode_i8mma_ws_bytes(n_seq, heads, head_dim, max_len));
    return b;
}


template <int D, bool I8>
static int launch_decode_t(const DecodeLaunch &L) {
    using namespace attn;
    DecodeParams p;
    const long long eh = (long long)L.n_seq * L.heads;
    p.chunk = decode_chunk(L.max_len, eh);
    p.max_splits = (L.max_len + p.chunk - 1) / p.chunk;
    // workspace: [tickets | part_ml | part_o], each 256-byte aligned.  The
    // tickets are cleared on the stream before every launch, so a workspace
    // may be shared by calls of any shape (ordered on one stream).
    char *ws = static_cast<char *>(L.ws);
    const size_t t_bytes = ((size_t)eh * sizeof(unsigned) + 255) / 256 * 256;
    const size_t ml_bytes = ((size_t)eh * p.max_splits * 2 * sizeof(float) + 255) / 256 * 256;
    p.tickets = reinterpret_cast<unsigned *>(ws);
    p.part_ml = reinterpret_cast<float *>(ws + t_bytes);
    p.part_o = reinterpret_cast<float *>(ws + t_bytes + ml_bytes);
    if (p.max_splits > 1) {
        cudaError_t e = cudaMemsetAsync(p.tickets, 0, (size_t)eh * sizeof(unsigned), L.stream);
        if (e != cudaSuccess) return set_error(ATTN_ERR_CUDA, "decode: ticket clear: %s", cudaGetErrorString(e));
    }
    p.q = L.q; p.kbase = L.kbase; p.vbase = L.vbase; p.kptrs = L.kptrs; p.vptrs = L.vptrs;
    p.ksbase = L.ksbase; p.vsbase = L.vsbase; p.ksptrs = L.ksptrs; p.vsptrs = L.vsptrs;
    p.lens = L.lens; p.out = L.out; p.err = L.err;
    p.row_stride = L.row_stride; p.cap = L.cap; p.H = L.heads; p.max_len = L.max_len;
    p.qscale = kLog2e / sqrtf((float)D);
    dim3 grid(p.max_splits, L.heads, L.n_seq);
    size_t smem = (size_t)(p.chunk + RowSlice<D, I8>::ROWS * D) * sizeof(float);
    return check_pdl(launch_pdl(decode_split_kernel<D, I8>, grid, dim3(kDecThreads), smem, L.stream, p),
                     "decode_split_kernel");
}

bool ensure_smem_attr(const void *func, size_t bytes);

template <int D, int CPL>
static int launch_rows_i8_t(const DecodeLaunch &L) {
    using namespace attn;
    DecodeParams p;
    p.chunk = rows_chunk(L.max_len, L.n_seq);
    p.max_splits = (L.max_len + p.chunk - 1) / p.chunk;
    const int H = L.heads, HD = H * D;
    // workspace: [tickets (n_seq) | part_ml | part_o], 256-byte aligned regions
    char *ws = static_cast<char *>(L.ws);
    const size_t t_bytes = ((size_t)L.n_seq * sizeof(unsigned) + 255) / 256 * 256;
    const size_t ml_bytes = ((size_t)L.n_seq * p.max_splits * H * 2 * sizeof(float) + 255) / 256 * 256;
    p.tickets = reinterpret_cast<unsigned *>(ws);
    p.part_ml = reinterpret_cast<float *>(ws + t_bytes);
    p.part_o = reinterpret_cast<float *>(ws + t_bytes + ml_bytes);
    if (p.max_splits > 1) {
        cudaError_t e = cudaMemsetAsync(p.tickets, 0, (size_t)L.n_seq * sizeof(unsigned), L.stream);
        if (e != cudaSuccess) return set_error(ATTN_ERR_CUDA, "decode: ticket clear: %s", cudaGetErrorString(e));
    }
    p.q = L.q; p.kbase = L.kbase; p.vbase = L.vbase; p.kptrs = L.kptrs; p.vptrs = L.vptrs;
    p.ksbase = L.ksbase; p.vsbase = L.vsbase; p.ksptrs = L.ksptrs; p.vsptrs = L.vsptrs;
    p.lens = L.lens; p.out = L.out; p.err = L.err;
    p.row_stride = L.row_stride; p.cap = L.cap; p.H = H; p.max_len = L.max_len;
    p.qscale = kLog2e / sqrtf((float)D);
    const size_t smem = (size_t)(H * p.chunk + kRowWarps * HD + 2 * H) * sizeof(float);
    if (!ensure_smem_attr((const void *)decode_rows_i8_kernel<D, CPL>, smem))
        return set_error(ATTN_ERR_CUDA, "decode: cannot set shared-memory size");
    cudaFuncSetAttribute(decode_rows_i8_kernel<D, CPL>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    dim3 grid(p.max_splits, L.n_seq);
    decode_rows_i8_kernel<D, CPL><<<grid, kRowWarps * 32, smem, L.stream>>>(p);
    return check_launch("decode_rows_i8_kernel");
}

static int launch_rows_i8(const DecodeLaunch &L) {
    const int cpl = L.heads * L.head_dim / 512;
    switch (L.head_dim * 10 + cpl) {
        case 321: return launch_rows_i8_t<32, 1>(L);
        case 322: return launch_rows_i8_t<32, 2>(L);
        case 324: return launch_rows_i8_t<32, 4>(L);
        case 641: return launch_rows_i8_t<64, 1>(L);
        case 642: return launch_rows_i8_t<64, 2>(L);
        case 644: return launch_rows_i8_t<64, 4>(L);
        case 1281: return launch_rows_i8_t<128, 1>(L);
        case 1282: return launch_rows_i8_t<128, 2>(L);
        case 1284: return launch_rows_i8_t<128, 4>(L);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "decode: no rows kernel for H*d=%d", L.heads * L.head_dim);
    }
}

bool decode_stream_ok(const DecodeLaunch &L);
bool decode_stream_shape_ok(int heads, int head_dim, int kv_dtype);
size_t decode_stream_ws_bytes(int n_seq, int heads, int head_dim, int max_len);
int launch_decode_stream(const DecodeLaunch &L);
bool decode_i8mma_ok(const DecodeLaunch &L);
int launch_decode_i8mma(const DecodeLaunch &L);

bool decode_ring_ok(const DecodeLaunch &L);
int launch_decode_ring(const DecodeLaunch &L);
bool decode_head_ok(const DecodeLaunch &L);
int launch_decode_head(const DecodeLaunch &L);

int launch_decode(const DecodeLaunch &L) {
    const bool i8 = L.kv_dtype == ATTN_I8;
    if (decode_head_ok(L)) return launch_decode_head(L);
    if (decode_ring_ok(L)) return launch_decode_ring(L);
    if (decode_i8mma_ok(L)) return launch_decode_i8mma(L);
    if (decode_stream_ok(L)) return launch_decode_stream(L);
    if (rows_i8_ok(L.heads, L.head_dim, L.kv_dtype)) return launch_rows_i8(L);
    switch (L.head_dim) {
        case 32: return i8 ? launch_decode_t<32, true>(L) : launch_decode_t<32, false>(L);
        case 64: return i8 ? launch_decode_t<64, true>(L) : launch_decode_t<64, false>(L);
        case 96: return i8 ? launch_decode_t<96, true>(L) : launch_decode_t<96, false>(L);
        case 128: return i8 ? launch_decode_t<128, true>(L) : launch_decode_t<128, false>(L);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "decode: head_dim %d not in {32,64,96,128}", L.head_dim);
    }
}

}  // namespace attn_host
