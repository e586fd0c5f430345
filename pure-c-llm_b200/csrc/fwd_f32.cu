// fwd_f32.cu -- causal flash forward with fp32 arithmetic (CUDA-core FFMA).
//
// Semantics: attention_forward, train.c:339-370 -- per (b, h) and query row i,
// softmax over keys j <= i of (q_i . k_j) / sqrt(d), then the weighted sum of
// v_j.  Instead of the reference's T x T probability matrix the kernel keeps
// a running max / sum per row (online softmax) and saves
// lse_i = max + log(sum), from which the backward rebuilds P exactly.
//
// One CTA per (64-row query tile, head, batch); query tiles are issued
// longest-first (the causal triangle makes tile i cost i+1 key tiles).  Key
// and value tiles are double-buffered with cp.async.
#include "flash_f32.cuh"

namespace attn {

struct FwdParams {
    const void *q, *k, *v;
    void *o;
    float *lse;
    long long in_stride, out_stride;
    int B, H, T;
    float qk_scale;            // log2(e) / sqrt(d)
};

template <typename T, int D>
__global__ void __launch_bounds__(kFThreads)
flash_fwd_f32_kernel(const FwdParams p)
{
    constexpr int TF = FTile<D>::FLOATS;
    extern __shared__ __align__(16) float sm[];
    float *Qs = sm;                    // [64][LD]
    float *Ks = Qs + TF;               // 2 x [64][LD]
    float *Vs = Ks + 2 * TF;           // 2 x [64][LD]
    float *Pt = Vs + 2 * TF;           // [64][68], weights transposed

    const int n_qt = (p.T + kFBM - 1) / kFBM;
    const int qt = n_qt - 1 - blockIdx.x;      // heaviest tiles first
    const int h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;
    const int q0 = qt * kFBM;

    const T *qg = static_cast<const T *>(p.q) + (long long)b * p.T * p.in_stride + (long long)h * D;
    const T *kg = static_cast<const T *>(p.k) + (long long)b * p.T * p.in_stride + (long long)h * D;
    const T *vg = static_cast<const T *>(p.v) + (long long)b * p.T * p.in_stride + (long long)h * D;

    load_tile<T, D>(Qs, qg, p.in_stride, q0, p.T, tid);
    load_tile<T, D>(Ks, kg, p.in_stride, 0, p.T, tid);
    load_tile<T, D>(Vs, vg, p.in_stride, 0, p.T, tid);
    cp_async_commit();

    float o[4][D / 8];
    float m[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY; l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < D / 8; c++) o[i][c] = 0.f;
    }

    for (int kt = 0; kt <= qt; kt++) {
        const int buf = kt & 1;
        if (kt < qt) {   // prefetch the next key/value tile into the other buffer
            load_tile<T, D>(Ks + (buf ^ 1) * TF, kg, p.in_stride, (kt + 1) * kFBN, p.T, tid);
            load_tile<T, D>(Vs + (buf ^ 1) * TF, vg, p.in_stride, (kt + 1) * kFBN, p.T, tid);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();

        float s[4][8];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) s[i][j] = 0.f;
        tile_qkT<D>(s, Qs, Ks + buf * TF, ty, tx);

        const bool diag = (kt == qt);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int row = ty + 16 * i;
            float mt = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float x = s[i][j] * p.qk_scale;
                if (diag && (tx + 8 * j) > row) x = -INFINITY;
                s[i][j] = x;
                mt = fmaxf(mt, x);
            }
            mt = row_max8(mt);
            const float mnew = fmaxf(m[i], mt);
            const float alpha = exp2f(m[i] - mnew);     // 0 on the first tile
            m[i] = mnew;
            float ls = 0.f;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float e = exp2f(s[i][j] - mnew);
                s[i][j] = e;
                ls += e;
            }
            l[i] = l[i] * alpha + row_sum8(ls);
#pragma unroll
            for (int c = 0; c < D / 8; c++) o[i][c] *= alpha;
        }
        store_weights_T(Pt, s, ty, tx);
        __syncthreads();
        tile_wM<D>(o, Pt, Vs + buf * TF, ty, tx);
        __syncthreads();   // Pt and this K/V buffer are rewritten next iteration
    }

    // epilogue: normalise and store
    T *og = static_cast<T *>(p.o) + (long long)b * p.T * p.out_stride + (long long)h * D;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int row = q0 + ty + 16 * i;
        if (row >= p.T) continue;
        const float inv = 1.f / l[i];
#pragma unroll
        for (int c = 0; c < D / 32; c++) {
            float4 v4 = make_float4(o[i][4 * c] * inv, o[i][4 * c + 1] * inv,
                                    o[i][4 * c + 2] * inv, o[i][4 * c + 3] * inv);
            store4(og + (long long)row * p.out_stride + 4 * tx + 32 * c, v4);
        }
        if (p.lse && tx == 0)
            p.lse[((long long)b * p.H + h) * p.T + row] = (m[i] + log2f(l[i])) * kLn2;
    }
}

}  // namespace attn

namespace attn_host {

bool ensure_smem_attr(const void *func, size_t bytes);

template <typename T, int D>
static int launch_fwd_f32_t(const attn::FwdParams &p, cudaStream_t s) {
    using namespace attn;
    const size_t smem = (size_t)(5 * FTile<D>::FLOATS + kFBN * (kFBM + 4)) * sizeof(float);
    if (!ensure_smem_attr((const void *)flash_fwd_f32_kernel<T, D>, smem))
        return set_error(ATTN_ERR_CUDA, "fwd_f32: cannot set shared-memory size");
    dim3 grid((p.T + kFBM - 1) / kFBM, p.H, p.B);
    flash_fwd_f32_kernel<T, D><<<grid, kFThreads, smem, s>>>(p);
    return check_launch("flash_fwd_f32_kernel");
}

int launch_fwd_f32(int dtype, int D, const void *q, const void *k, const void *v, void *o,
                   float *lse, long long in_stride, long long out_stride, int B, int H, int T,
                   cudaStream_t s)
{
    attn::FwdParams p;
    p.q = q; p.k = k; p.v = v; p.o = o; p.lse = lse;
    p.in_stride = in_stride; p.out_stride = out_stride;
    p.B = B; p.H = H; p.T = T;
    p.qk_scale = attn::kLog2e / sqrtf((float)D);
    const bool bf = dtype == ATTN_BF16;
    switch (D) {
        case 32: return bf ? launch_fwd_f32_t<__nv_bfloat16, 32>(p, s) : launch_fwd_f32_t<float, 32>(p, s);
        case 64: return bf ? launch_fwd_f32_t<__nv_bfloat16, 64>(p, s) : launch_fwd_f32_t<float, 64>(p, s);
        case 96: return bf ? launch_fwd_f32_t<__nv_bfloat16, 96>(p, s) : launch_fwd_f32_t<float, 96>(p, s);
        case 128: return bf ? launch_fwd_f32_t<__nv_bfloat16, 128>(p, s) : launch_fwd_f32_t<float, 128>(p, s);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "fwd: head_dim %d not in {32,64,96,128}", D);
    }
}

}  // namespace attn_host
