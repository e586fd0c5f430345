// kv.cu -- INT8 cache quantiser, cache row append, and the head-shard permute
// used after a multi-GPU all-gather.
#include "common.cuh"

namespace attn {

// One warp per (row, head).  Bit-exact restatement of the reference's
// symmetric absmax quantiser (gemm_bench.c:225-236) at (row, head)
// granularity: amax = max(1e-8, max|x|) (the reference seeds amax with 1e-8
// and keeps the larger value), scale = amax / 127, inv = 1 / scale (both IEEE
// round-to-nearest divisions -- this file is built without fast-math), and
// code = lroundf(x * inv) (half away from zero) clamped to [-127, 127].
template <int D>
__global__ void quantize_int8_kernel(const float *__restrict__ x, long long rows, int heads,
                                     long long row_stride, int8_t *__restrict__ codes,
                                     float *__restrict__ scales)
{
    constexpr int E = D / 32;
    const long long unit = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (unit >= rows * heads) return;
    const int lane = threadIdx.x & 31;
    const long long r = unit / heads;
    const int h = (int)(unit % heads);
    const float *src = x + r * row_stride + (long long)h * D;
    int8_t *dst = codes + r * row_stride + (long long)h * D;
    float v[E];
    float amax = 1e-8f;
#pragma unroll
    for (int i = 0; i < E; i++) {
        v[i] = src[lane + 32 * i];
        amax = fmaxf(amax, fabsf(v[i]));
    }
    amax = warp_max(amax);
    const float scale = __fdiv_rn(amax, 127.0f);
    const float inv = __fdiv_rn(1.0f, scale);
#pragma unroll
    for (int i = 0; i < E; i++) {
        float t = roundf(__fmul_rn(v[i], inv));
        t = fminf(127.f, fmaxf(-127.f, t));
        dst[lane + 32 * i] = (int8_t)(int)t;
    }
    if (lane == 0) scales[r * heads + h] = scale;
}

// Copies one token's K/V row (fp32) into row `pos` of an fp32 cache.
__global__ void append_f32_kernel(const float *__restrict__ krow, const float *__restrict__ vrow,
                                  float *__restrict__ kdst, float *__restrict__ vdst, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) { kdst[i] = krow[i]; vdst[i] = vrow[i]; }
}

// staging [G][B][T][Hg][D]  ->  out (B*T, H*D) with H = G*Hg.
template <typename T>
__global__ void gather_permute_kernel(const T *__restrict__ staging, T *__restrict__ out,
                                      int G, int B, int Tn, int Hg, int D)
{
    const long long total = (long long)G * B * Tn * Hg * D;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        long long t = i;
        const int c = (int)(t % D); t /= D;
        const int hg = (int)(t % Hg); t /= Hg;
        const int tok = (int)(t % Tn); t /= Tn;
        const int b = (int)(t % B); t /= B;
        const int g = (int)t;
        const long long o = ((long long)b * Tn + tok) * ((long long)G * Hg * D) + ((long long)g * Hg + hg) * D + c;
        out[o] = staging[i];
    }
}

}  // namespace attn

namespace attn_host {

int launch_quantize_int8(const float *x, long long rows, int heads, int head_dim,
                         long long row_stride, int8_t *codes, float *scales, cudaStream_t s)
{
    using namespace attn;
    const long long units = rows * heads;
    if (units == 0) return ATTN_OK;
    const int warps = 8;
    const unsigned blocks = (unsigned)((units + warps - 1) / warps);
    switch (head_dim) {
        case 32: quantize_int8_kernel<32><<<blocks, warps * 32, 0, s>>>(x, rows, heads, row_stride, codes, scales); break;
        case 64: quantize_int8_kernel<64><<<blocks, warps * 32, 0, s>>>(x, rows, heads, row_stride, codes, scales); break;
        case 96: quantize_int8_kernel<96><<<blocks, warps * 32, 0, s>>>(x, rows, heads, row_stride, codes, scales); break;
        case 128: quantize_int8_kernel<128><<<blocks, warps * 32, 0, s>>>(x, rows, heads, row_stride, codes, scales); break;
        default: return set_error(ATTN_ERR_UNSUPPORTED, "quantize: head_dim %d not in {32,64,96,128}", head_dim);
    }
    return check_launch("quantize_int8_kernel");
}

int launch_append_f32(const float *krow, const float *vrow, float *kdst, float *vdst, int n,
                      cudaStream_t s)
{
    attn::append_f32_kernel<<<(n + 255) / 256, 256, 0, s>>>(krow, vrow, kdst, vdst, n);
    return check_launch("append_f32_kernel");
}

int launch_gather_permute(const void *staging, void *out, int G, int B, int T, int H, int D,
                          int dtype, cudaStream_t s)
{
    const int Hg = H / G;
    const long long total = (long long)B * T * H * D;
    const unsigned blocks = (unsigned)std::min<long long>((total + 255) / 256, 148LL * 16);
    if (dtype == ATTN_F32)
        attn::gather_permute_kernel<float><<<blocks, 256, 0, s>>>(
            static_cast<const float *>(staging), static_cast<float *>(out), G, B, T, Hg, D);
    else
        attn::gather_permute_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
            static_cast<const __nv_bfloat16 *>(staging), static_cast<__nv_bfloat16 *>(out), G, B, T, Hg, D);
    return check_launch("gather_permute_kernel");
}

}  // namespace attn_host
