// decode_head.cu -- KV-cached decode attention over an fp32 cache with one
// CTA per (sequence, head), for calls with few sequences and short caches
// (the 16-layer generator step).
//
// Semantics: cached_attention, transformer.c:203-248 -- for every head, one
// query row scores cache rows 0..len-1 with (q . k_j) / sqrt(d), softmaxes
// them and sums the value rows.
//
// A generator step reads ~40 MB: ~6 us at the HBM roof, so what matters is
// keeping bytes in flight from the first microsecond and adding no second
// pass, merge or launch.  Each CTA owns every cache row of one (sequence,
// head) -- the head's d floats of each token row, one 128-512 byte piece per
// row -- so no CTA waits for or merges with another and the call needs no
// workspace.  The CTA streams its pieces through a ring of shared-memory
// stages with cp.async (K and V of R rows per stage, S stages in flight) and
// consumes each stage in one pass: lane groups of d/4 lanes take one row
// each (16-byte pieces), reduce the dot product with shuffles and keep an
// online softmax (running max, sum, weighted value sum) per group; the
// groups and warps combine at the end.
#include <algorithm>

#include "common.cuh"
#include "decode_launch.cuh"
#include "sm100.cuh"

namespace attn {
namespace dh {

#ifndef ATTN_DH_ROWS
#define ATTN_DH_ROWS 32
#endif
#ifndef ATTN_DH_MAX_STAGES
#define ATTN_DH_MAX_STAGES 12
#endif
constexpr int kThreads = 128;
constexpr int kRows = ATTN_DH_ROWS;   // rows per stage
// Stages in the ring: up to ATTN_DH_MAX_STAGES, at most 128 KB of shared memory.
// At d 32 (the C1 shape, 8 KB stages) 12 stages keep 88 KB in flight per CTA
// and still let two CTAs share an SM: 3.80 TB/s per generator step, against
// 3.52 with 8 stages and 2.44 with 16 (one CTA per SM); 48- and 64-row stages
// of the same depth in bytes ran at 3.68-3.77.
template <int D> __host__ __device__ constexpr int stages() {
    return 128 * 1024 / (2 * kRows * D * 4) < ATTN_DH_MAX_STAGES ? 128 * 1024 / (2 * kRows * D * 4)
                                                                  : ATTN_DH_MAX_STAGES;
}

struct Params {
    const float *q;                   // n_seq x row elements (head h at h*D)
    const char *kbase, *vbase;        // contiguous caches (kptrs == nullptr)
    const void *const *kptrs, *const *vptrs;
    const int *lens;                  // n_seq, device; NULL = max_len for all
    float *out;                       // n_seq x H*D
    int *err;
    long long row_bytes_stride;       // bytes between cache rows
    long long cap;                    // rows per sequence (contiguous layout)
    int H, max_len;
    float qscale;                     // log2(e) / sqrt(D)
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int D>
__global__ void __launch_bounds__(kThreads)
decode_head_kernel(const __grid_constant__ Params p)
{
    constexpr int LPR = D / 4;                        // lanes per row (16 bytes each)
    constexpr int RPI = 32 / LPR;                     // rows per warp instruction
    constexpr int STAGE_F = 2 * kRows * D;            // floats of one stage (K rows, then V rows)
    constexpr int CHUNKS = STAGE_F / 4 / kThreads;    // 16-byte copies per thread per stage
    constexpr int kStages = stages<D>();
    static_assert(CHUNKS >= 1 && (STAGE_F / 4) % kThreads == 0, "stage geometry");
    extern __shared__ float4 ring4[];
    float *ring = reinterpret_cast<float *>(ring4);
    __shared__ float red_m[kThreads / LPR], red_l[kThreads / LPR];
    __shared__ float red_o[kThreads / LPR][D];

    // the work before this call on the stream may be writing the cache: the
    // CTAs of a programmatic launch become resident early and wait here
    pdl_begin();
    const int h = blockIdx.x, e = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane / LPR, sub = lane % LPR;
    const char *kb, *vb;
    if (p.kptrs) {
        kb = static_cast<const char *>(p.kptrs[e]);
        vb = static_cast<const char *>(p.vptrs[e]);
    } else {
        kb = p.kbase + (long long)e * p.cap * p.row_bytes_stride;
        vb = p.vbase + (long long)e * p.cap * p.row_bytes_stride;
    }
    int len = p.lens ? __ldg(p.lens + e) : p.max_len;
    const float4 q4 = __ldg(reinterpret_cast<const float4 *>(p.q + (long long)e * p.H * D + h * D) + sub);
    if (len < 1 || len > p.max_len) {
        if (h == 0 && tid == 0) atomicExch(p.err, 0x100 + (len < 1 ? 1 : 2));
        len = len < 1 ? 1 : p.max_len;
    }
    if ((((uintptr_t)kb | (uintptr_t)vb) & 15) != 0) {   // misaligned slab: nothing is read
        if (tid == 0) atomicExch(p.err, 0x340);
        len = 0;
    }
    const int n_st = (len + kRows - 1) / kRows;
    kb += (long long)h * D * 4;
    vb += (long long)h * D * 4;
    const uint32_t ring_s = sm100::smem_u32(ring);
    // stage s: copy c of this thread = piece (row, 16-byte column) of K or V
    auto issue = [&](int s) {
        if (s < n_st) {
            const uint32_t dst0 = ring_s + (uint32_t)((s % kStages) * STAGE_F) * 4u;
#pragma unroll
            for (int c = 0; c < CHUNKS; c++) {
                const int idx = c * kThreads + tid;       // 16-byte piece of the stage
                const int isv = idx >= kRows * LPR;
                const int pr = isv ? idx - kRows * LPR : idx;
                const int r = pr / LPR, col = pr % LPR;
                const int row = s * kRows + r;
                if (row < len) {
                    const char *src = (isv ? vb : kb) + (long long)row * p.row_bytes_stride + col * 16;
                    cp_async16(dst0 + (uint32_t)idx * 16u, src);
                }
            }
        }
        cp_async_commit();                            // (empty groups keep the count uniform)
    };
#pragma unroll
    for (int s = 0; s < kStages - 1; s++) issue(s);

    const float qs = p.qscale;
    const float4 qv = make_float4(q4.x * qs, q4.y * qs, q4.z * qs, q4.w * qs);
    float m = -INFINITY, l = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < n_st; s++) {
        issue(s + kStages - 1);
        cp_async_wait<kStages - 1>();                 // stage s has landed (this thread's copies)
        __syncthreads();                              // ... and every thread's
        const float *st = ring + (s % kStages) * STAGE_F;
        // this warp's rows of the stage: warp w takes rows w*RW .. w*RW + RW - 1
        constexpr int RW = kRows / (kThreads / 32);
#pragma unroll
        for (int i = 0; i < RW / RPI; i++) {
            const int r = warp * RW + i * RPI + grp;
            const int row = s * kRows + r;
            const float4 k4 = *reinterpret_cast<const float4 *>(st + r * D + sub * 4);
            const float4 v4 = *reinterpret_cast<const float4 *>(st + kRows * D + r * D + sub * 4);
            float a = qv.x * k4.x;
            a = fmaf(qv.y, k4.y, a);
            a = fmaf(qv.z, k4.z, a);
            a = fmaf(qv.w, k4.w, a);
#pragma unroll
            for (int off = LPR / 2; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
            if (row < len) {                          // uniform within the lane group
                if (a > m) {
                    const float f = sm100::ex2(m - a);    // 0 on the group's first row
                    l *= f;
                    o.x *= f; o.y *= f; o.z *= f; o.w *= f;
                    m = a;
                }
                const float pr = sm100::ex2(a - m);
                l += pr;
                o.x = fmaf(pr, v4.x, o.x);
                o.y = fmaf(pr, v4.y, o.y);
                o.z = fmaf(pr, v4.z, o.z);
                o.w = fmaf(pr, v4.w, o.w);
            }
        }
        __syncthreads();                              // the stage may be refilled
    }
    cp_async_wait<0>();
    // combine the lane groups (one state per group of LPR lanes) in shared memory
    const int g = tid / LPR;
    if (sub == 0) {
        red_m[g] = m;
        red_l[g] = l;
    }
    *reinterpret_cast<float4 *>(&red_o[g][sub * 4]) = o;
    __syncthreads();
    if (tid < D) {
        constexpr int G = kThreads / LPR;
        float M = -INFINITY;
#pragma unroll
        for (int i = 0; i < G; i++) M = fmaxf(M, red_m[i]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int i = 0; i < G; i++) {
            const float f = red_m[i] == -INFINITY ? 0.f : sm100::ex2(red_m[i] - M);
            L += red_l[i] * f;
            O += red_o[i][tid] * f;
        }
        p.out[(long long)e * p.H * D + h * D + tid] = len > 0 ? O / L : 0.f;
    }
}

}  // namespace dh
}  // namespace attn

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace attn_host {

bool ensure_smem_attr(const void *func, size_t bytes);

// fp32 caches, at most 512 (sequence, head) units -- about one wave of CTAs
// -- and at most 1024 cached rows, so that one CTA streaming a whole unit
// finishes about as soon as the HBM delivers the call's bytes; bigger calls
// go to the kernels that split rows over CTAs.
bool decode_head_ok(const DecodeLaunch &L) {
    if (L.kv_dtype != ATTN_F32) return false;
    if (L.head_dim != 32 && L.head_dim != 64 && L.head_dim != 128) return false;
    if ((L.row_stride * 4) % 16 || ((uintptr_t)L.q & 15)) return false;
    if (!L.kptrs && (((uintptr_t)L.kbase | (uintptr_t)L.vbase) & 15)) return false;
    const long long units = (long long)L.n_seq * L.heads;
    return units <= 512 && L.max_len <= 1024;
}

template <int D>
static int launch_head_t(const DecodeLaunch &L) {
    using namespace attn::dh;
    Params p;
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
    p.H = L.heads;
    p.max_len = L.max_len;
    p.qscale = attn::kLog2e / sqrtf((float)D);
    const size_t smem = (size_t)stages<D>() * 2 * kRows * D * sizeof(float);
    if (!ensure_smem_attr((const void *)decode_head_kernel<D>, smem))
        return set_error(ATTN_ERR_CUDA, "decode: cannot set shared-memory size");
    // a programmatic dependent of the work before it on the stream (see the kernel)
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(L.heads, L.n_seq);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = L.stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, decode_head_kernel<D>, p);
    if (e != cudaSuccess) return set_error(ATTN_ERR_CUDA, "decode_head_kernel: %s", cudaGetErrorString(e));
    return ATTN_OK;
}

int launch_decode_head(const DecodeLaunch &L) {
    switch (L.head_dim) {
        case 32: return launch_head_t<32>(L);
        case 64: return launch_head_t<64>(L);
        case 128: return launch_head_t<128>(L);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "decode: no per-head kernel for head_dim %d", L.head_dim);
    }
}

}  // namespace attn_host
