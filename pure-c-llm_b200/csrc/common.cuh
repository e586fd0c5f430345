// common.cuh -- small shared helpers for the attention kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "attn_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libattn_b200 is written for sm_100a (B200) only"
#endif

namespace attn {

// log2(e): scores are kept in the base-2 domain so the softmax uses exp2.
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// --- element loads into fp32 -------------------------------------------------
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

// Loads 4 consecutive elements (16 B of fp32 or 8 B of bf16) as floats.
__device__ __forceinline__ float4 load4(const float *p) {
    return __ldg(reinterpret_cast<const float4 *>(p));
}
__device__ __forceinline__ float4 load4(const __nv_bfloat16 *p) {
    uint2 u = __ldg(reinterpret_cast<const uint2 *>(p));
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162 *>(&u.x);
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162 *>(&u.y);
    float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
}
__device__ __forceinline__ void store4(float *p, float4 v) {
    *reinterpret_cast<float4 *>(p) = v;
}
__device__ __forceinline__ void store4(__nv_bfloat16 *p, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t *>(&a);
    u.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = u;
}
__device__ __forceinline__ float4 load4_cg(const float *p) {
    return __ldcg(reinterpret_cast<const float4 *>(p));
}

// First statement of a kernel launched by launch_pdl: lets the next kernel on
// the stream be scheduled, then waits until the work before this grid has
// finished and its memory is visible (the CTAs may start early).
__device__ __forceinline__ void pdl_begin() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace attn

// Host-side launch status helper shared by the .cu files of the library.
namespace attn_host {
int set_error(int status, const char *fmt, ...);

// Launches `kernel` as a programmatic dependent of the work before it on the
// stream (the kernel begins with pdl_begin): its CTAs may become resident
// while that work finishes, which hides most of the launch gap between
// back-to-back kernels.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}
inline int check_pdl(cudaError_t e, const char *what) {
    if (e != cudaSuccess) return set_error(ATTN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return ATTN_OK;
}
inline int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ATTN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return ATTN_OK;
}
}  // namespace attn_host
