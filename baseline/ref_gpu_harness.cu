// ref_gpu_harness.cu -- builds the reference's own GPU attention, the
// cuBLAS-SGEMM path of gpu_kernels.cu (attn_fwd 403-435, attn_bwd 438-489,
// k_causal_softmax 264-280, k_softmax_bwd 283-295), at a chosen shape, and
// its gemm_nn (112-120), as GPU baselines for the benchmark.  Nothing of it
// is used by the library.
//
// The reference fixes its shape with unconditional macros (gpu_kernels.h:17-31)
// behind an include guard, so this harness includes the header first, replaces
// the shape macros with REF_B / REF_H / REF_T / REF_D from the command line,
// and then compiles the unmodified gpu_kernels.cu (whose own #include of the
// header is skipped by the guard).
#include "gpu_kernels.h"

#undef DIM
#undef N_HEADS
#undef D_HEAD
#undef MAX_SEQ_LEN
#undef B_SIZE
#undef T_SIZE
#undef M_ROWS
#define DIM (REF_H * REF_D)
#define N_HEADS REF_H
#define D_HEAD REF_D
#define MAX_SEQ_LEN REF_T
#define B_SIZE REF_B
#define T_SIZE MAX_SEQ_LEN
#define M_ROWS (B_SIZE * T_SIZE)

#include "gpu_kernels.cu"

extern "C" {
// the compiled-in shape
void refgpu_shape(int *b, int *h, int *t, int *d) {
    *b = B_SIZE;
    *h = N_HEADS;
    *t = T_SIZE;
    *d = D_HEAD;
}
void refgpu_init(void) { gpu_init(); }
void refgpu_attn_fwd(const float *Q, const float *K, const float *V, float *att, float *probs) {
    attn_fwd(Q, K, V, att, probs);
}
/* gemm_nn (gpu_kernels.cu:112-120): C = A B (+ bias), row-major fp32, the
 * call train_kaggle.cu:152-154 makes for each of Q, K and V. */
void refgpu_gemm_nn(const float *A, const float *B, const float *bias, float *C, int M, int K, int N) {
    gemm_nn(A, B, bias, C, M, K, N);
}
void refgpu_attn_bwd(float *dQ, float *dK, float *dV, float *scratch, const float *dAtt, const float *Q,
                     const float *K, const float *V, const float *probs) {
    attn_bwd(dQ, dK, dV, scratch, dAtt, Q, K, V, probs);
}
}
