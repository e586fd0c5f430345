/*
 * attn_oracle.c -- CPU restatement of pure-c-llm's causal attention, used ONLY
 * as test infrastructure (the parity checker for the CUDA library and the
 * timed CPU baseline of bench.py).  Nothing in the product links this file.
 *
 * Parity pin: every routine here is checked against the reference's own
 * attention, compiled from the unmodified reference sources into
 * oracle/_ref/ (see oracle/Makefile), through the committed fixtures in
 * tests/golden/ (tests/test_oracle.py).
 *
 * Shapes are runtime arguments (the reference fixes them with macros).  The
 * activation layout is the reference's: a (rows x row_stride) row-major float
 * matrix, head h of token t at [t*row_stride + h*head_dim, +head_dim)
 * (transformer.h:15-18).  row_stride is heads*head_dim for the training
 * tensors (train.c uses D_MODEL).
 *
 * Arithmetic order follows the reference loop by loop so that, compiled with
 * the same flags, results agree to the last few ulps:
 *   - dot product accumulated in d order, scaled AFTER the dot
 *     (train.c:352-353, transformer.c:216-223);
 *   - running max seeded with -1e30 (train.c:349);
 *   - expf(s - max), sum in j order, normalised by multiplying with 1/sum
 *     (train.c:356-359);
 *   - output accumulated in j order (train.c:361-367).
 * Double-precision twins of forward and decode are the tie-breakers.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------
 * Causal forward for B sequences of T tokens, H heads of size d.
 * Follows attention_forward, train.c:339-370.  `probs` (B*H*T*T, may be
 * NULL) receives the normalised probabilities exactly like the reference;
 * `lse` (B*H*T, may be NULL) receives max + log(sum) of the scaled scores,
 * the per-row statistic the CUDA path saves instead of probs.
 * ---------------------------------------------------------------------- */
ORACLE_API void oracle_attn_forward(const float *q, const float *k, const float *v,
                                    float *att, float *probs, float *lse,
                                    int B, int T, int H, int d, long row_stride)
{
    const float scale = 1.0f / sqrtf((float)d);
    float *row = (float *)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
    for (int bh = 0; bh < B * H; bh++) {
        const int b = bh / H, h = bh % H;
        const long off = (long)h * d;
        for (int i = 0; i < T; i++) {
            const float *qi = q + (size_t)(b * T + i) * row_stride + off;
            float mx = -1e30f;
            for (int j = 0; j <= i; j++) {
                const float *kj = k + (size_t)(b * T + j) * row_stride + off;
                float acc = 0.0f;
                for (int c = 0; c < d; c++) acc += qi[c] * kj[c];
                acc *= scale;
                row[j] = acc;
                if (acc > mx) mx = acc;
            }
            float sum = 0.0f;
            for (int j = 0; j <= i; j++) {
                float e = expf(row[j] - mx);
                row[j] = e;
                sum += e;
            }
            const float inv = 1.0f / sum;
            for (int j = 0; j <= i; j++) row[j] *= inv;
            if (lse) lse[(size_t)bh * T + i] = mx + logf(sum);
            if (probs) {
                float *p = probs + ((size_t)bh * T + i) * T;
                memcpy(p, row, sizeof(float) * (size_t)(i + 1));
                for (int j = i + 1; j < T; j++) p[j] = 0.0f;
            }
            float *oi = att + (size_t)(b * T + i) * row_stride + off;
            for (int c = 0; c < d; c++) oi[c] = 0.0f;
            for (int j = 0; j <= i; j++) {
                const float pj = row[j];
                const float *vj = v + (size_t)(b * T + j) * row_stride + off;
                for (int c = 0; c < d; c++) oi[c] += pj * vj[c];
            }
        }
    }
    free(row);
}

/* Same forward in double precision (tie-breaker), output rounded to float. */
ORACLE_API void oracle_attn_forward_f64(const float *q, const float *k, const float *v,
                                        float *att, int B, int T, int H, int d,
                                        long row_stride)
{
    const double scale = 1.0 / sqrt((double)d);
    double *row = (double *)malloc(sizeof(double) * (size_t)(T > 0 ? T : 1));
    double *o = (double *)malloc(sizeof(double) * (size_t)d);
    for (int bh = 0; bh < B * H; bh++) {
        const int b = bh / H, h = bh % H;
        const long off = (long)h * d;
        for (int i = 0; i < T; i++) {
            const float *qi = q + (size_t)(b * T + i) * row_stride + off;
            double mx = -1e300;
            for (int j = 0; j <= i; j++) {
                const float *kj = k + (size_t)(b * T + j) * row_stride + off;
                double acc = 0.0;
                for (int c = 0; c < d; c++) acc += (double)qi[c] * (double)kj[c];
                row[j] = acc * scale;
                if (row[j] > mx) mx = row[j];
            }
            double sum = 0.0;
            for (int j = 0; j <= i; j++) { row[j] = exp(row[j] - mx); sum += row[j]; }
            for (int c = 0; c < d; c++) o[c] = 0.0;
            for (int j = 0; j <= i; j++) {
                const float *vj = v + (size_t)(b * T + j) * row_stride + off;
                for (int c = 0; c < d; c++) o[c] += row[j] * (double)vj[c];
            }
            float *oi = att + (size_t)(b * T + i) * row_stride + off;
            for (int c = 0; c < d; c++) oi[c] = (float)(o[c] / sum);
        }
    }
    free(o);
    free(row);
}

/* ------------------------------------------------------------------------
 * Analytic backward, follows attention_backward, train.c:373-407.
 * ACCUMULATES into dq/dk/dv like the reference (callers zero them first,
 * train.c:561-563).  `probs` is the B*H*T*T output of the forward.
 * ---------------------------------------------------------------------- */
ORACLE_API void oracle_attn_backward(float *dq, float *dk, float *dv, const float *d_att,
                                     const float *q, const float *k, const float *v,
                                     const float *probs, int B, int T, int H, int d,
                                     long row_stride)
{
    const float scale = 1.0f / sqrtf((float)d);
    float *dprobs = (float *)malloc(sizeof(float) * (size_t)(T > 0 ? T : 1));
    for (int bh = 0; bh < B * H; bh++) {
        const int b = bh / H, h = bh % H;
        const long off = (long)h * d;
        for (int i = 0; i < T; i++) {
            const float *dao = d_att + (size_t)(b * T + i) * row_stride + off;
            const float *p = probs + ((size_t)bh * T + i) * T;
            for (int j = 0; j <= i; j++) {
                const float *vj = v + (size_t)(b * T + j) * row_stride + off;
                float *dvj = dv + (size_t)(b * T + j) * row_stride + off;
                float dp = 0.0f;
                for (int c = 0; c < d; c++) { dp += dao[c] * vj[c]; dvj[c] += p[j] * dao[c]; }
                dprobs[j] = dp;
            }
            float dot = 0.0f;
            for (int j = 0; j <= i; j++) dot += p[j] * dprobs[j];
            float *dqi = dq + (size_t)(b * T + i) * row_stride + off;
            const float *qi = q + (size_t)(b * T + i) * row_stride + off;
            for (int j = 0; j <= i; j++) {
                const float ds = p[j] * (dprobs[j] - dot) * scale;
                const float *kj = k + (size_t)(b * T + j) * row_stride + off;
                float *dkj = dk + (size_t)(b * T + j) * row_stride + off;
                for (int c = 0; c < d; c++) { dqi[c] += ds * kj[c]; dkj[c] += ds * qi[c]; }
            }
        }
    }
    free(dprobs);
}

/* ------------------------------------------------------------------------
 * KV-cached decode for one query token, follows cached_attention,
 * transformer.c:203-248: attends cache rows 0..pos of every head.  The cache
 * rows are `row_stride` floats apart (D_MODEL in the reference).
 * ---------------------------------------------------------------------- */
ORACLE_API void oracle_cached_attention(const float *q, const float *kcache,
                                        const float *vcache, float *out, int pos,
                                        int H, int d, long row_stride)
{
    const float scale = 1.0f / sqrtf((float)d);
    float *srow = (float *)malloc(sizeof(float) * (size_t)(pos + 1));
    for (int h = 0; h < H; h++) {
        const long off = (long)h * d;
        const float *qh = q + off;
        float mx = -1e30f;
        for (int j = 0; j <= pos; j++) {
            const float *kj = kcache + (size_t)j * row_stride + off;
            float acc = 0.0f;
            for (int c = 0; c < d; c++) acc += qh[c] * kj[c];
            acc *= scale;
            srow[j] = acc;
            if (acc > mx) mx = acc;
        }
        float sum = 0.0f;
        for (int j = 0; j <= pos; j++) { float e = expf(srow[j] - mx); srow[j] = e; sum += e; }
        const float inv = 1.0f / sum;
        for (int j = 0; j <= pos; j++) srow[j] *= inv;
        float *oh = out + off;
        for (int c = 0; c < d; c++) oh[c] = 0.0f;
        for (int j = 0; j <= pos; j++) {
            const float pj = srow[j];
            const float *vj = vcache + (size_t)j * row_stride + off;
            for (int c = 0; c < d; c++) oh[c] += pj * vj[c];
        }
    }
    free(srow);
}

/* Double-precision decode twin (tie-breaker). */
ORACLE_API void oracle_cached_attention_f64(const float *q, const float *kcache,
                                            const float *vcache, float *out, int pos,
                                            int H, int d, long row_stride)
{
    const double scale = 1.0 / sqrt((double)d);
    double *srow = (double *)malloc(sizeof(double) * (size_t)(pos + 1));
    for (int h = 0; h < H; h++) {
        const long off = (long)h * d;
        double mx = -1e300;
        for (int j = 0; j <= pos; j++) {
            double acc = 0.0;
            for (int c = 0; c < d; c++)
                acc += (double)q[off + c] * (double)kcache[(size_t)j * row_stride + off + c];
            srow[j] = acc * scale;
            if (srow[j] > mx) mx = srow[j];
        }
        double sum = 0.0;
        for (int j = 0; j <= pos; j++) { srow[j] = exp(srow[j] - mx); sum += srow[j]; }
        for (int c = 0; c < d; c++) {
            double o = 0.0;
            for (int j = 0; j <= pos; j++) o += srow[j] * (double)vcache[(size_t)j * row_stride + off + c];
            out[off + c] = (float)(o / sum);
        }
    }
    free(srow);
}

/* ------------------------------------------------------------------------
 * INT8 KV quantiser.  The scheme is the reference's symmetric absmax
 * quantiser, quantize_A in gemm_bench.c:225-236 (amax floored at 1e-8,
 * scale = amax/127, q = lroundf(x * (1/scale)) clamped to [-127, 127]),
 * applied per (token, head) over head_dim elements instead of per tensor.
 * The +128 offset of gemm_bench.c:233 exists only for VNNI's u8 x s8 form
 * and is not part of the stored cache; codes are signed.
 * ---------------------------------------------------------------------- */
ORACLE_API void oracle_quantize_kv_int8(const float *x, int8_t *codes, float *scales,
                                        long rows, int H, int d, long row_stride)
{
    for (long r = 0; r < rows; r++) {
        for (int h = 0; h < H; h++) {
            const float *src = x + (size_t)r * row_stride + (size_t)h * d;
            int8_t *dst = codes + (size_t)r * row_stride + (size_t)h * d;
            float amax = 1e-8f;
            for (int c = 0; c < d; c++) { float a = fabsf(src[c]); if (a > amax) amax = a; }
            const float scale = amax / 127.0f, inv = 1.0f / scale;
            for (int c = 0; c < d; c++) {
                int qv = (int)lroundf(src[c] * inv);
                qv = qv > 127 ? 127 : (qv < -127 ? -127 : qv);
                dst[c] = (int8_t)qv;
            }
            scales[(size_t)r * H + h] = scale;
        }
    }
}

/* Dequantise a cache back to float: x = code * scale (per token, head). */
ORACLE_API void oracle_dequantize_kv_int8(const int8_t *codes, const float *scales, float *x,
                                          long rows, int H, int d, long row_stride)
{
    for (long r = 0; r < rows; r++)
        for (int h = 0; h < H; h++) {
            const float s = scales[(size_t)r * H + h];
            for (int c = 0; c < d; c++) {
                const size_t i = (size_t)r * row_stride + (size_t)h * d + c;
                x[i] = (float)codes[i] * s;
            }
        }
}

/* ------------------------------------------------------------------------
 * out(M,N) = in(M,K) @ W(K,N) + bias(N), rows of `in` ldx apart: the
 * reference's matmul_forward (train.c:181-211) in its portable i-k-j order
 * (train.c:193-205: out row zeroed, then out[n] += in[k] * W[k][n] for k in
 * order), the bias added after the product (train.c:206-212).  train.c:517-519
 * and train_kaggle.cu:152-154 apply it to a layer's Q, K and V projections.
 * `bias` may be NULL.  The double-precision twin is the tie-breaker.
 * ---------------------------------------------------------------------- */
ORACLE_API void oracle_matmul_forward(float *out, const float *in, const float *W, const float *bias,
                                      int M, int K, int N, long ldx)
{
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        float *o = out + (size_t)m * N;
        const float *x = in + (size_t)m * ldx;
        for (int n = 0; n < N; n++) o[n] = 0.0f;
        for (int k = 0; k < K; k++) {
            const float a = x[k];
            const float *wr = W + (size_t)k * N;
            for (int n = 0; n < N; n++) o[n] += a * wr[n];
        }
        if (bias)
            for (int n = 0; n < N; n++) o[n] += bias[n];
    }
}

ORACLE_API void oracle_matmul_forward_f64(double *out, const float *in, const float *W, const float *bias,
                                          int M, int K, int N, long ldx)
{
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++) {
        double *o = out + (size_t)m * N;
        const float *x = in + (size_t)m * ldx;
        for (int n = 0; n < N; n++) o[n] = 0.0;
        for (int k = 0; k < K; k++) {
            const double a = x[k];
            const float *wr = W + (size_t)k * N;
            for (int n = 0; n < N; n++) o[n] += a * (double)wr[n];
        }
        if (bias)
            for (int n = 0; n < N; n++) o[n] += bias[n];
    }
}
