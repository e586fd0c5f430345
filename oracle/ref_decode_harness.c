/*
 * ref_decode_harness.c -- exposes the reference's OWN KV-cached decode
 * attention (static cached_attention, transformer.c:203-248) and its B=1
 * prefill attention (multihead_attention, transformer.c:58-107) from the
 * unmodified reference source, for the parity checker only.
 *
 * transformer.h fixes T_MAX/D_MODEL/N_HEADS with unguarded macros
 * (transformer.h:35-39), so this file stands in for that header: it defines
 * its include guard, the shape macros from -DREF_* flags, and the three
 * struct types transformer.c dereferences (field names as declared at
 * transformer.h:45-103), then includes transformer.c from the reference
 * tree.  tensor.c is compiled alongside from the reference tree as well.
 */
#define TRANSFORMER_H 1
#define T_MAX   REF_T_MAX
#define D_MODEL REF_D_MODEL
#define N_HEADS REF_N_HEADS
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

void multihead_attention(const float *Q, const float *K, const float *V,
                         float *out, float *scores, int T);
void forward_block(float *x, const LayerWeights *w, DecodeScratch *s,
                   float *kcache, float *vcache, int pos);
void forward_layer(float *x, const LayerWeights *w, LayerScratch *s, int T);

#include "transformer.c"

#define REF_API __attribute__((visibility("default")))

/* scores: N_HEADS * T_MAX floats of scratch, as DecodeScratch.scores. */
REF_API void ref_cached_attention(const float *q, const float *kcache, const float *vcache,
                                  float *out, float *scores, int pos)
{
    cached_attention(q, kcache, vcache, out, scores, pos);
}

/* scores: N_HEADS * T * T floats of scratch, as LayerScratch.scores. */
REF_API void ref_multihead_attention(const float *Q, const float *K, const float *V,
                                     float *out, float *scores, int T)
{
    multihead_attention(Q, K, V, out, scores, T);
}

REF_API int ref_d_model(void) { return D_MODEL; }
REF_API int ref_n_heads(void) { return N_HEADS; }
REF_API int ref_t_max(void) { return T_MAX; }
