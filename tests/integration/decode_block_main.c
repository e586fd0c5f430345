/*
 * decode_block_main.c -- the reference's own KV-cached decoder block,
 * forward_block (transformer.c:251-285), run for 16 layers x 128 tokens at
 * the C1 decode shape (d_model 512 = 16 heads x 32, 512 cached rows before
 * the first token).  The Makefile builds it twice from the unmodified
 * reference sources: as they are (the CPU reference), and with the attention
 * call of forward_block (transformer.c:266) routed to the library's
 * attn_cached_attention_host, the one-line edit a maintainer makes.  Both
 * write the residual vector after every token to the file named on the
 * command line, so a test can compare the runs.
 *
 * transformer.h fixes its shapes with unguarded macros (transformer.h:35-39),
 * so this file stands in for the header (its include guard, the shapes and
 * the struct types transformer.c dereferences, field names as declared at
 * transformer.h:45-103) before including the transformer source.
 */
#define TRANSFORMER_H 1
#define T_MAX   640
#define D_MODEL 512
#define N_HEADS 16
#define D_HEAD  (D_MODEL / N_HEADS)
#define D_FF    (4 * D_MODEL)

typedef struct {
    float *Wq, *Wk, *Wv, *bq, *bk, *bv, *Wo, *bo;
    float *ln1_gamma, *ln1_beta, *ln2_gamma, *ln2_beta;
    float *W_ff1, *b_ff1, *W_ff2, *b_ff2;
} LayerWeights;
typedef struct {
    float *ln, *Q, *K, *V, *attn, *proj, *scores, *ff_hidden, *ff_out;
} LayerScratch;
typedef struct {
    float *ln, *q, *attn, *proj, *scores, *ff_hidden, *ff_out;
} DecodeScratch;

void multihead_attention(const float *Q, const float *K, const float *V, float *out, float *scores, int T);
void forward_block(float *x, const LayerWeights *w, DecodeScratch *s, float *kcache, float *vcache, int pos);
void forward_layer(float *x, const LayerWeights *w, LayerScratch *s, int T);

#ifdef ROUTED
#include "attn_b200.h"
#endif
#include TRANSFORMER_SRC

#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#define LAYERS 16
#define PRIOR 512
#define STEPS 128

/* splitmix64 -> Box-Muller normals (the generator of the repository's synth.py) */
static uint64_t g_state = 2024;
static double uniform01(void) {
    uint64_t z = (g_state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}
static float normal(float std) {
    const double u1 = 1.0 - uniform01(), u2 = uniform01();
    return (float)(std * sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2));
}
static float *filled(size_t n, float std, float mean) {
    float *p = (float *)malloc(n * sizeof(float));
    if (!p) { fprintf(stderr, "out of memory\n"); exit(1); }
    for (size_t i = 0; i < n; i++) p[i] = mean + (std > 0 ? normal(std) : 0.0f);
    return p;
}

int main(int argc, char **argv) {
    if (argc < 2) { fprintf(stderr, "usage: %s out.bin\n", argv[0]); return 2; }
#ifdef ROUTED
    if (attn_set_decode_macro_shape(N_HEADS, D_HEAD, T_MAX) != ATTN_OK) {
        fprintf(stderr, "%s\n", attn_last_error());
        return 1;
    }
#endif
    LayerWeights w[LAYERS];
    float *kc[LAYERS], *vc[LAYERS];
    for (int l = 0; l < LAYERS; l++) {
        w[l].Wq = filled((size_t)D_MODEL * D_MODEL, 0.05f, 0);
        w[l].Wk = filled((size_t)D_MODEL * D_MODEL, 0.05f, 0);
        w[l].Wv = filled((size_t)D_MODEL * D_MODEL, 0.05f, 0);
        w[l].Wo = filled((size_t)D_MODEL * D_MODEL, 0.02f, 0);
        w[l].bq = filled(D_MODEL, 0.02f, 0);
        w[l].bk = filled(D_MODEL, 0.02f, 0);
        w[l].bv = filled(D_MODEL, 0.02f, 0);
        w[l].bo = filled(D_MODEL, 0.02f, 0);
        w[l].ln1_gamma = filled(D_MODEL, 0.1f, 1.0f);
        w[l].ln1_beta = filled(D_MODEL, 0.1f, 0);
        w[l].ln2_gamma = filled(D_MODEL, 0.1f, 1.0f);
        w[l].ln2_beta = filled(D_MODEL, 0.1f, 0);
        w[l].W_ff1 = filled((size_t)D_MODEL * D_FF, 0.02f, 0);
        w[l].b_ff1 = filled(D_FF, 0.02f, 0);
        w[l].W_ff2 = filled((size_t)D_FF * D_MODEL, 0.02f, 0);
        w[l].b_ff2 = filled(D_MODEL, 0.02f, 0);
        kc[l] = filled((size_t)T_MAX * D_MODEL, 1.0f, 0);      /* rows >= PRIOR are overwritten */
        vc[l] = filled((size_t)T_MAX * D_MODEL, 1.0f, 0);
    }
    DecodeScratch s;
    s.ln = filled(D_MODEL, 0, 0);
    s.q = filled(D_MODEL, 0, 0);
    s.attn = filled(D_MODEL, 0, 0);
    s.proj = filled(D_MODEL, 0, 0);
    s.scores = filled((size_t)N_HEADS * T_MAX, 0, 0);
    s.ff_hidden = filled(D_FF, 0, 0);
    s.ff_out = filled(D_MODEL, 0, 0);
    float *x = filled(D_MODEL, 1.0f, 0);
    FILE *f = fopen(argv[1], "wb");
    if (!f) { perror(argv[1]); return 1; }
    for (int t = 0; t < STEPS; t++) {
        for (int i = 0; i < D_MODEL; i++) x[i] = normal(1.0f);     /* this token's embedding */
        for (int l = 0; l < LAYERS; l++) forward_block(x, &w[l], &s, kc[l], vc[l], PRIOR + t);
        fwrite(x, sizeof(float), D_MODEL, f);
        fwrite(s.attn, sizeof(float), D_MODEL, f);             /* the last layer's attention output */
    }
    fclose(f);
    return 0;
}
