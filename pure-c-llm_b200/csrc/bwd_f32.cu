// bwd_f32.cu -- causal flash backward with fp32 arithmetic (CUDA-core FFMA).
//
// Semantics: attention_backward, train.c:373-407 (and gpu_kernels.cu:438-489):
//   dv_j += sum_i p_ij dO_i
//   dp_ij = dO_i . v_j
//   ds_ij = p_ij (dp_ij - D_i) / sqrt(d),  D_i = sum_j p_ij dp_ij = dO_i . O_i
//   dq_i += sum_j ds_ij k_j,   dk_j += sum_i ds_ij q_i
// P is rebuilt from the forward's saved lse (p_ij = exp(s_ij - lse_i)) instead
// of a stored T x T matrix.  Three deterministic kernels, no atomics:
//   1. rowdot:  D_i = dO_i . O_i  (and lse converted to base 2), per row
//   2. dkdv:    one CTA per 64-row key tile, loops over the query tiles i >= j
//   3. dq:      one CTA per 64-row query tile, loops over the key tiles j <= i
#include "flash_f32.cuh"

namespace attn {

struct BwdParams {
    const void *q, *k, *v, *o, *dout;
    const float *lse;          // [B][H][T], natural log
    float *lse2;               // workspace [B][H][T]: lse * log2(e)
    float *dvec;               // workspace [B][H][T]: D_i
    void *dq, *dk, *dv;
    long long in_stride, out_stride;
    int B, H, T, accumulate;
    float qk_scale;            // log2(e) / sqrt(d)
    float ds_scale;            // 1 / sqrt(d)
};

template <typename T, int D>
__global__ void bwd_rowdot_kernel(const BwdParams p)
{
    // one warp per (row, head); grid covers B*T*H warps
    const long long unit = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const long long total = (long long)p.B * p.T * p.H;
    if (unit >= total) return;
    const int lane = threadIdx.x & 31;
    const int h = (int)(unit % p.H);
    const long long bt = unit / p.H;
    const int b = (int)(bt / p.T), t = (int)(bt % p.T);
    const T *o = static_cast<const T *>(p.o) + bt * p.out_stride + (long long)h * D;
    const T *g = static_cast<const T *>(p.dout) + bt * p.in_stride + (long long)h * D;
    float acc = 0.f;
#pragma unroll
    for (int c = lane; c < D; c += 32) acc = fmaf(to_f32(o[c]), to_f32(g[c]), acc);
    acc = warp_sum(acc);
    if (lane == 0) {
        const long long r = ((long long)b * p.H + h) * p.T + t;
        p.dvec[r] = acc;
        p.lse2[r] = p.lse[r] * kLog2e;
    }
}

// The same statistics, one block per 32 consecutive rows of one (batch, head):
// 8 threads per row, each reading D/8 contiguous elements of O and dO with
// 8-byte loads (a row's 8 threads cover it in one contiguous segment), a
// 3-step shuffle sum, and coalesced writes of the 32 rows' D and lse2 (which
// are laid out [B][H][T]).  Needs 8-byte aligned rows.
template <typename T, int D>
__global__ void __launch_bounds__(256) bwd_rowdot_tile_kernel(const BwdParams p)
{
    pdl_begin();   // launched by launch_pdl
    static_assert(D % 32 == 0, "8 threads x a multiple of 4 elements per row");
    constexpr int EP = D / 8;                        // elements per thread
    const int row = threadIdx.x >> 3, part = threadIdx.x & 7;
    const int t = (int)blockIdx.x * 32 + row, h = (int)blockIdx.y, b = (int)blockIdx.z;
    float acc = 0.f;
    if (t < p.T) {
        const long long bt = (long long)b * p.T + t;
        const T *o = static_cast<const T *>(p.o) + bt * p.out_stride + (long long)h * D + part * EP;
        const T *g = static_cast<const T *>(p.dout) + bt * p.in_stride + (long long)h * D + part * EP;
        if constexpr (sizeof(T) == 4) {
#pragma unroll
            for (int c = 0; c < EP; c += 2) {
                const float2 x = __ldg(reinterpret_cast<const float2 *>(o + c));
                const float2 y = __ldg(reinterpret_cast<const float2 *>(g + c));
                acc = fmaf(x.x, y.x, acc);
                acc = fmaf(x.y, y.y, acc);
            }
        } else {
#pragma unroll
            for (int c = 0; c < EP; c += 4) {           // 4 bf16 = two 32-bit words
                const uint2 x = __ldg(reinterpret_cast<const uint2 *>(o + c));
                const uint2 y = __ldg(reinterpret_cast<const uint2 *>(g + c));
                acc = fmaf(__uint_as_float(x.x << 16), __uint_as_float(y.x << 16), acc);
                acc = fmaf(__uint_as_float(x.x & 0xffff0000u), __uint_as_float(y.x & 0xffff0000u), acc);
                acc = fmaf(__uint_as_float(x.y << 16), __uint_as_float(y.y << 16), acc);
                acc = fmaf(__uint_as_float(x.y & 0xffff0000u), __uint_as_float(y.y & 0xffff0000u), acc);
            }
        }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    if (part == 0 && t < p.T) {
        const long long r = ((long long)b * p.H + h) * p.T + t;
        p.dvec[r] = acc;
        p.lse2[r] = p.lse[r] * kLog2e;
    }
}

template <int D> struct BwdCfg {
    static constexpr int NBUF = D <= 96 ? 2 : 1;   // double-buffer streamed tiles when smem allows
};

template <typename T>
__device__ __forceinline__ void store_row4(T *dst, float4 v, bool acc) {
    if (acc) {
        float4 old = load4(dst);
        v.x += old.x; v.y += old.y; v.z += old.z; v.w += old.w;
    }
    store4(dst, v);
}

// ---- dK, dV: one CTA per key tile ------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(kFThreads)
bwd_dkdv_kernel(const BwdParams p)
{
    pdl_begin();   // launched by launch_pdl
    constexpr int TF = FTile<D>::FLOATS;
    constexpr int NB = BwdCfg<D>::NBUF;
    extern __shared__ __align__(16) float sm[];
    float *Ks = sm;
    float *Vs = Ks + TF;
    float *Qs = Vs + TF;             // NB x [64][LD]
    float *Gs = Qs + NB * TF;        // NB x [64][LD]  (dO)
    float *W1 = Gs + NB * TF;        // [64][68]  P^T weights
    float *W2 = W1 + kFBN * (kFBM + 4);   // [64][68]  dS^T weights
    float *rowv = W2 + kFBN * (kFBM + 4); // NB x [2][64]: lse2, D of the query tile

    const int n_t = (p.T + kFBM - 1) / kFBM;
    const int kt = n_t - 1 - blockIdx.x;   // blockIdx 0 -> last key tile (fewest query tiles)
    const int h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;
    const int k0 = kt * kFBN;
    const long long base_in = (long long)b * p.T * p.in_stride + (long long)h * D;
    const T *qg = static_cast<const T *>(p.q) + base_in;
    const T *kg = static_cast<const T *>(p.k) + base_in;
    const T *vg = static_cast<const T *>(p.v) + base_in;
    const T *gg = static_cast<const T *>(p.dout) + base_in;
    const float *lse2 = p.lse2 + ((long long)b * p.H + h) * p.T;
    const float *dv_ = p.dvec + ((long long)b * p.H + h) * p.T;

    auto stage_q = [&](int qt, int buf) {
        load_tile<T, D>(Qs + buf * TF, qg, p.in_stride, qt * kFBM, p.T, tid);
        load_tile<T, D>(Gs + buf * TF, gg, p.in_stride, qt * kFBM, p.T, tid);
        if (tid < kFBM) {
            const int r = qt * kFBM + tid;
            rowv[buf * 128 + tid] = r < p.T ? lse2[r] : 0.f;
            rowv[buf * 128 + 64 + tid] = r < p.T ? dv_[r] : 0.f;
        }
    };

    load_tile<T, D>(Ks, kg, p.in_stride, k0, p.T, tid);
    load_tile<T, D>(Vs, vg, p.in_stride, k0, p.T, tid);
    stage_q(kt, 0);
    cp_async_commit();

    float dk[4][D / 8], dvv[4][D / 8];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int c = 0; c < D / 8; c++) { dk[i][c] = 0.f; dvv[i][c] = 0.f; }

    for (int qt = kt; qt < n_t; qt++) {
        const int buf = NB == 2 ? ((qt - kt) & 1) : 0;
        if (NB == 2 && qt + 1 < n_t) {
            stage_q(qt + 1, buf ^ 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float *Qb = Qs + buf * TF, *Gb = Gs + buf * TF, *rv = rowv + buf * 128;
        const bool diag = (qt == kt);

        // S^T (key rows ty+16i, query cols tx+8j) -> P^T
        float s[4][8];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) s[i][j] = 0.f;
        tile_qkT<D>(s, Ks, Qb, ty, tx);
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int kr = ty + 16 * i, qc = tx + 8 * j;
                float e = exp2f(s[i][j] * p.qk_scale - rv[qc]);
                if (diag && qc < kr) e = 0.f;
                if (qt * kFBM + qc >= p.T) e = 0.f;
                s[i][j] = e;
            }
        store_weights_T(W1, s, ty, tx);

        // dP^T = V dO^T, then dS^T = P^T (dP^T - D) / sqrt(d)
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) s[i][j] = 0.f;
        tile_qkT<D>(s, Vs, Gb, ty, tx);
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int qc = tx + 8 * j;
                const float pw = W1[qc * (kFBM + 4) + 4 * ty + i];   // own entry, no sync needed
                s[i][j] = pw * (s[i][j] - rv[64 + qc]) * p.ds_scale;
            }
        store_weights_T(W2, s, ty, tx);
        __syncthreads();

        tile_wM<D>(dvv, W1, Gb, ty, tx);
        tile_wM<D>(dk, W2, Qb, ty, tx);
        __syncthreads();
        if (NB == 1 && qt + 1 < n_t) { stage_q(qt + 1, 0); cp_async_commit(); }
    }

    T *dkg = static_cast<T *>(p.dk) + (long long)b * p.T * p.out_stride + (long long)h * D;
    T *dvg = static_cast<T *>(p.dv) + (long long)b * p.T * p.out_stride + (long long)h * D;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int row = k0 + ty + 16 * i;
        if (row >= p.T) continue;
#pragma unroll
        for (int c = 0; c < D / 32; c++) {
            const long long off = (long long)row * p.out_stride + 4 * tx + 32 * c;
            store_row4(dkg + off, make_float4(dk[i][4 * c], dk[i][4 * c + 1], dk[i][4 * c + 2], dk[i][4 * c + 3]), p.accumulate);
            store_row4(dvg + off, make_float4(dvv[i][4 * c], dvv[i][4 * c + 1], dvv[i][4 * c + 2], dvv[i][4 * c + 3]), p.accumulate);
        }
    }
}

// ---- dQ: one CTA per query tile --------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(kFThreads)
bwd_dq_kernel(const BwdParams p)
{
    pdl_begin();   // launched by launch_pdl
    constexpr int TF = FTile<D>::FLOATS;
    constexpr int NB = BwdCfg<D>::NBUF;
    extern __shared__ __align__(16) float sm[];
    float *Qs = sm;
    float *Gs = Qs + TF;
    float *Ks = Gs + TF;             // NB x tile
    float *Vs = Ks + NB * TF;        // NB x tile
    float *W = Vs + NB * TF;         // [64][68] dS weights

    const int n_t = (p.T + kFBM - 1) / kFBM;
    const int qt = n_t - 1 - blockIdx.x;
    const int h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;
    const int q0 = qt * kFBM;
    const long long base_in = (long long)b * p.T * p.in_stride + (long long)h * D;
    const T *qg = static_cast<const T *>(p.q) + base_in;
    const T *kg = static_cast<const T *>(p.k) + base_in;
    const T *vg = static_cast<const T *>(p.v) + base_in;
    const T *gg = static_cast<const T *>(p.dout) + base_in;
    const float *lse2 = p.lse2 + ((long long)b * p.H + h) * p.T;
    const float *dv_ = p.dvec + ((long long)b * p.H + h) * p.T;

    load_tile<T, D>(Qs, qg, p.in_stride, q0, p.T, tid);
    load_tile<T, D>(Gs, gg, p.in_stride, q0, p.T, tid);
    load_tile<T, D>(Ks, kg, p.in_stride, 0, p.T, tid);
    load_tile<T, D>(Vs, vg, p.in_stride, 0, p.T, tid);
    cp_async_commit();

    float rl[4], rd[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = q0 + ty + 16 * i;
        rl[i] = r < p.T ? lse2[r] : 0.f;
        rd[i] = r < p.T ? dv_[r] : 0.f;
    }
    float dq[4][D / 8];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int c = 0; c < D / 8; c++) dq[i][c] = 0.f;

    for (int kt = 0; kt <= qt; kt++) {
        const int buf = NB == 2 ? (kt & 1) : 0;
        if (NB == 2 && kt < qt) {
            load_tile<T, D>(Ks + (buf ^ 1) * TF, kg, p.in_stride, (kt + 1) * kFBN, p.T, tid);
            load_tile<T, D>(Vs + (buf ^ 1) * TF, vg, p.in_stride, (kt + 1) * kFBN, p.T, tid);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float *Kb = Ks + buf * TF, *Vb = Vs + buf * TF;
        const bool diag = (kt == qt);

        float s[4][8], dp[4][8];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) { s[i][j] = 0.f; dp[i][j] = 0.f; }
        tile_qkT<D>(s, Qs, Kb, ty, tx);
        tile_qkT<D>(dp, Gs, Vb, ty, tx);
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int qr = ty + 16 * i, kc = tx + 8 * j;
                float e = exp2f(s[i][j] * p.qk_scale - rl[i]);
                if (diag && kc > qr) e = 0.f;
                s[i][j] = e * (dp[i][j] - rd[i]) * p.ds_scale;
            }
        store_weights_T(W, s, ty, tx);
        __syncthreads();
        tile_wM<D>(dq, W, Kb, ty, tx);
        __syncthreads();
        if (NB == 1 && kt < qt) {
            load_tile<T, D>(Ks, kg, p.in_stride, (kt + 1) * kFBN, p.T, tid);
            load_tile<T, D>(Vs, vg, p.in_stride, (kt + 1) * kFBN, p.T, tid);
            cp_async_commit();
        }
    }

    T *dqg = static_cast<T *>(p.dq) + (long long)b * p.T * p.out_stride + (long long)h * D;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int row = q0 + ty + 16 * i;
        if (row >= p.T) continue;
#pragma unroll
        for (int c = 0; c < D / 32; c++)
            store_row4(dqg + (long long)row * p.out_stride + 4 * tx + 32 * c,
                       make_float4(dq[i][4 * c], dq[i][4 * c + 1], dq[i][4 * c + 2], dq[i][4 * c + 3]),
                       p.accumulate);
    }
}

}  // namespace attn

namespace attn_host {

bool ensure_smem_attr(const void *func, size_t bytes);

// Row statistics through the tiled kernel when the rows are 8-byte aligned,
// else through the warp-per-row kernel.
template <typename T, int D>
static int launch_rowdot_t(const attn::BwdParams &p, cudaStream_t s) {
    const bool aligned = ((((uintptr_t)p.o | (uintptr_t)p.dout) & 7) == 0) &&
                         (p.in_stride * (long long)sizeof(T)) % 8 == 0 && (p.out_stride * (long long)sizeof(T)) % 8 == 0;
    if (aligned && p.H <= 65535 && p.B <= 65535) {
        const dim3 grid((unsigned)((p.T + 31) / 32), (unsigned)p.H, (unsigned)p.B);
        const int st = check_pdl(launch_pdl(attn::bwd_rowdot_tile_kernel<T, D>, grid, dim3(256), 0, s, p),
                                 "bwd_rowdot_tile_kernel");
        if (st) return st;
    } else {
        const long long rows = (long long)p.B * p.T * p.H;
        attn::bwd_rowdot_kernel<T, D><<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(p);
    }
    return check_launch("bwd_rowdot_kernel");
}

// Row statistics for any backward: lse2 = lse * log2(e) and D = dO . O per
// (b, h, t), into the workspace (shared with the tensor-core backward).
int launch_bwd_rowdot(int dtype, int D, const void *o, const void *dout, const float *lse, float *ws,
                      long long in_stride, long long out_stride, int B, int H, int T, cudaStream_t s) {
    attn::BwdParams p;
    p.o = o; p.dout = dout; p.lse = lse;
    p.lse2 = ws;
    p.dvec = ws + (long long)B * H * T;
    p.in_stride = in_stride; p.out_stride = out_stride;
    p.B = B; p.H = H; p.T = T;
    const bool bf = dtype == ATTN_BF16;
    switch (D) {
        case 32: return bf ? launch_rowdot_t<__nv_bfloat16, 32>(p, s) : launch_rowdot_t<float, 32>(p, s);
        case 64: return bf ? launch_rowdot_t<__nv_bfloat16, 64>(p, s) : launch_rowdot_t<float, 64>(p, s);
        case 96: return bf ? launch_rowdot_t<__nv_bfloat16, 96>(p, s) : launch_rowdot_t<float, 96>(p, s);
        case 128: return bf ? launch_rowdot_t<__nv_bfloat16, 128>(p, s) : launch_rowdot_t<float, 128>(p, s);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "bwd: head_dim %d", D);
    }
}

size_t bwd_f32_workspace_bytes(int B, int H, int T) {
    return (size_t)2 * B * H * T * sizeof(float) + 256;
}

template <typename T, int D>
static int launch_bwd_f32_t(const attn::BwdParams &p, cudaStream_t s) {
    using namespace attn;
    constexpr int TF = FTile<D>::FLOATS;
    constexpr int NB = BwdCfg<D>::NBUF;
    const size_t smem_kv = (size_t)((2 + 2 * NB) * TF + 2 * kFBN * (kFBM + 4) + NB * 128) * sizeof(float);
    const size_t smem_q = (size_t)((2 + 2 * NB) * TF + kFBN * (kFBM + 4)) * sizeof(float);
    if (!ensure_smem_attr((const void *)bwd_dkdv_kernel<T, D>, smem_kv) ||
        !ensure_smem_attr((const void *)bwd_dq_kernel<T, D>, smem_q))
        return set_error(ATTN_ERR_CUDA, "bwd_f32: cannot set shared-memory size");
    int st = launch_rowdot_t<T, D>(p, s);
    if (st) return st;
    dim3 grid((p.T + kFBM - 1) / kFBM, p.H, p.B);
    if ((st = check_pdl(launch_pdl(bwd_dkdv_kernel<T, D>, grid, dim3(kFThreads), smem_kv, s, p), "bwd_dkdv_kernel")))
        return st;
    return check_pdl(launch_pdl(bwd_dq_kernel<T, D>, grid, dim3(kFThreads), smem_q, s, p), "bwd_dq_kernel");
}

int launch_bwd_f32(int dtype, int D, const void *dout, const void *q, const void *k,
                   const void *v, const void *o, const float *lse, void *dq, void *dk, void *dv,
                   int accumulate, void *ws, long long in_stride, long long out_stride, int B,
                   int H, int T, cudaStream_t s)
{
    attn::BwdParams p;
    p.q = q; p.k = k; p.v = v; p.o = o; p.dout = dout; p.lse = lse;
    p.lse2 = static_cast<float *>(ws);
    p.dvec = p.lse2 + (long long)B * H * T;
    p.dq = dq; p.dk = dk; p.dv = dv;
    p.in_stride = in_stride; p.out_stride = out_stride;
    p.B = B; p.H = H; p.T = T; p.accumulate = accumulate;
    p.qk_scale = attn::kLog2e / sqrtf((float)D);
    p.ds_scale = 1.0f / sqrtf((float)D);
    const bool bf = dtype == ATTN_BF16;
    switch (D) {
        case 32: return bf ? launch_bwd_f32_t<__nv_bfloat16, 32>(p, s) : launch_bwd_f32_t<float, 32>(p, s);
        case 64: return bf ? launch_bwd_f32_t<__nv_bfloat16, 64>(p, s) : launch_bwd_f32_t<float, 64>(p, s);
        case 96: return bf ? launch_bwd_f32_t<__nv_bfloat16, 96>(p, s) : launch_bwd_f32_t<float, 96>(p, s);
        case 128: return bf ? launch_bwd_f32_t<__nv_bfloat16, 128>(p, s) : launch_bwd_f32_t<float, 128>(p, s);
        default: return set_error(ATTN_ERR_UNSUPPORTED, "bwd: head_dim %d not in {32,64,96,128}", D);
    }
}

}  // namespace attn_host
