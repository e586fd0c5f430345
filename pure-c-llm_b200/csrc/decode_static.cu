// decode_static.cu -- the KV-cached decode entry point that allocates nothing.
//
// Who needs it: callers that must not allocate device memory themselves or let
// a library do it -- a token-generation loop whose device memory is owned by
// another allocator (a fixed budget carved up in advance), or a
// latency-critical loop in which a cudaMalloc would implicitly synchronise the
// device.  attn_decode_ex needs a caller workspace or allocates its own on
// first use; this variant instead uses one fixed scratch array that lives in
// the library's device image, sized ATTN_DECODE_STATIC_SCRATCH_BYTES.
//
// The array is reserved on every GPU that loads the library, for as long as the
// process runs.  All calls share it and it keeps the last call's contents; the
// split-merge tickets that must start at zero are cleared on the stream at
// every call.  Two calls whose kernels overlap on the GPU (different streams,
// no ordering) race on the array.
#include <mutex>

#include "common.cuh"

static __device__ __align__(256) unsigned char g_decode_scratch[ATTN_DECODE_STATIC_SCRATCH_BYTES];

// In host code `g_decode_scratch` names a host-side stand-in, not device memory:
// the device address comes from cudaGetSymbolAddress, fetched once per device
// with that device current.
static void *scratch_address(int device) {
    static std::mutex mu;
    static void *addr[128] = {nullptr};
    if (device < 0 || device >= 128) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[device]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
        if (e != cudaSuccess) {
            attn_host::set_error(ATTN_ERR_CUDA, "attn_decode_static_ex: cudaGetSymbolAddress failed: %s",
                                 cudaGetErrorString(e));
            return nullptr;
        }
        addr[device] = p;
    }
    return addr[device];
}

extern "C" int attn_decode_static_ex(const attn_decode_shape *s, const float *q, const void *kcache,
                                     const void *vcache, const float *kscale, const float *vscale,
                                     const int *lens, float *out, attn_stream_t stream) {
    if (!s) return attn_host::set_error(ATTN_ERR_INVALID, "attn_decode_static_ex: shape is NULL");
    const size_t need = attn_decode_workspace_bytes(s);
    if (need > (size_t)ATTN_DECODE_STATIC_SCRATCH_BYTES)
        return attn_host::set_error(ATTN_ERR_WORKSPACE,
                                    "attn_decode_static_ex: n_seq=%d heads=%d head_dim=%d max_len=%d needs %zu "
                                    "bytes of scratch, above the fixed %u bytes; use attn_decode_ex",
                                    s->n_seq, s->heads, s->head_dim, s->max_len, need,
                                    (unsigned)ATTN_DECODE_STATIC_SCRATCH_BYTES);
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess)
        return attn_host::set_error(ATTN_ERR_CUDA, "attn_decode_static_ex: cudaGetDevice failed");
    void *scratch = scratch_address(device);
    if (!scratch) return ATTN_ERR_CUDA;
    return attn_decode_ex(s, q, kcache, vcache, kscale, vscale, lens, out, scratch,
                          (size_t)ATTN_DECODE_STATIC_SCRATCH_BYTES, stream);
}
