/*
 * ref_quant_harness.c -- exposes the reference's OWN INT8 quantiser
 * (static quantize_A, gemm_bench.c:225-236) from the unmodified source, for
 * the parity checker only.  Called on one (token, head) slice at a time
 * (M = 1, K = Kpad = head_dim) it is exactly the per-(token, head) absmax
 * scheme of the INT8 KV cache: it returns the scale and writes code + 128.
 */
#define main ref_gemm_main_unused
#include "gemm_bench.c"
#undef main

__attribute__((visibility("default")))
float ref_quantize_A(const float *A, uint8_t *Au, int M, int K, int Kpad)
{
    return quantize_A(A, Au, M, K, Kpad);
}
