// abi_cxx.cu -- the drop-in attn_fwd / attn_bwd again, with C++ linkage.
//
// gpu_kernels.h declares attn_fwd and attn_bwd (gpu_kernels.h:67-72) outside
// any extern "C" block, and the trainer is compiled by nvcc as CUDA C++
// (train_kaggle.cu), so an unchanged trainer refers to the C++-mangled names.
// These definitions export exactly those names; the C-linkage symbols of
// include/attn_b200.h serve C callers.  Both run the same code.
//
// This file must not include attn_b200.h: a C++ function may not share its
// name and parameter list with the header's extern "C" declaration in one
// translation unit.

namespace attn_host {
void dropin_fwd(const float *Q, const float *K, const float *V, float *att, float *probs);
void dropin_bwd(float *dQ, float *dK, float *dV, float *scratch, const float *dAtt, const float *Q,
                const float *K, const float *V, const float *probs);
}  // namespace attn_host

#define ATTN_CXX_API __attribute__((visibility("default")))

ATTN_CXX_API void attn_fwd(const float *Q, const float *K, const float *V, float *att, float *probs) {
    attn_host::dropin_fwd(Q, K, V, att, probs);
}

ATTN_CXX_API void attn_bwd(float *dQ, float *dK, float *dV, float *scratch, const float *dAtt, const float *Q,
                           const float *K, const float *V, const float *probs) {
    attn_host::dropin_bwd(dQ, dK, dV, scratch, dAtt, Q, K, V, probs);
}
