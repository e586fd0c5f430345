// decode_launch.cuh -- host-side description of one decode call, shared by the
// C ABI (abi.cu) and the decode launchers (decode.cu, decode_stream.cu).
#pragma once
#include <cuda_runtime.h>

namespace attn_host {

struct DecodeLaunch {
    int n_seq, heads, head_dim, kv_dtype, max_len;
    long long row_stride, cap;            // elements between cache rows; rows per sequence
    const float *q;
    const void *kbase, *vbase;            // contiguous caches (kptrs == nullptr)
    const void *const *kptrs, *const *vptrs;
    const float *ksbase, *vsbase;         // INT8 scales, contiguous layout
    const float *const *ksptrs, *const *vsptrs;
    const int *lens;
    float *out;
    void *ws;
    int *err;
    cudaStream_t stream;
};

}  // namespace attn_host
