// fwd_bf16_sm100.cu -- tcgen05/TMA flash forward for bf16 (placeholder until
// the tensor-core kernel lands; the bf16 path runs fwd_f32's bf16 variant).
#include "common.cuh"

namespace attn_host {
bool fwd_bf16_sm100_supported(int, long long, long long) { return false; }
int launch_fwd_bf16_sm100(int, const void *, const void *, const void *, void *, float *,
                          long long, long long, int, int, int, int *, cudaStream_t) {
    return set_error(ATTN_ERR_UNSUPPORTED, "bf16 tensor-core forward not built");
}
}  // namespace attn_host
