/*
 * ref_train_harness.c -- exposes the reference's OWN training attention
 * (static attention_forward / attention_backward, train.c:339-407) from the
 * unmodified reference source, for the parity checker only.  The source is
 * pulled in with #include from the reference tree at build time
 * (oracle/Makefile, REF=...); nothing of it is copied into this repository.
 *
 * Shapes are the reference's compile-time macros: build with
 * -DBLOCK_SIZE=<max T> -DD_MODEL=<H*d> -DN_HEADS=<H> (train.c:34-52 guards
 * them with #ifndef).  T may be any value <= BLOCK_SIZE at call time because
 * only the stack array dprobs[T_SIZE] (train.c:380) depends on the macro.
 */
#define main ref_train_main_unused
#include "train.c"
#undef main

#define REF_API __attribute__((visibility("default")))

REF_API void ref_attention_forward(const float *q, const float *k, const float *v,
                                   float *att, float *probs, int B, int T)
{
    attention_forward(q, k, v, att, probs, B, T);
}

/* Accumulates into dq/dk/dv exactly like the reference (train.c:372). */
REF_API void ref_attention_backward(float *dq, float *dk, float *dv, const float *d_att,
                                    const float *q, const float *k, const float *v,
                                    const float *probs, int B, int T)
{
    attention_backward(dq, dk, dv, d_att, q, k, v, probs, B, T);
}

REF_API int ref_d_model(void) { return D_MODEL; }
REF_API int ref_n_heads(void) { return N_HEADS; }
REF_API int ref_block_size(void) { return BLOCK_SIZE; }

/* out(M,N) = in(M,K) @ W(K,N) + bias(N): the reference's own matmul_forward
 * (train.c:181-211), which train.c:517-519 calls for the Q, K and V
 * projections of a layer. */
REF_API void ref_matmul_forward(float *out, const float *in, const float *W, const float *bias,
                                int M, int K, int N)
{
    matmul_forward(out, in, W, bias, M, K, N);
}
