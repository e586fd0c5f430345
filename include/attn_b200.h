/*
 * attn_b200.h -- C ABI of the B200 causal-attention engine (libattn_b200.so).
 *
 * Drop-in boundary for pure-c-llm's attention:
 *   - attn_fwd / attn_bwd keep the exact signatures, pointer meaning and
 *     error behaviour of gpu_kernels.h:67-72 (device pointers, shapes from
 *     compile-time-style defaults, void return, exit(1) on a CUDA error like
 *     CUDA_CHECK at gpu_kernels.h:34-36), so train_kaggle.cu:155/199 link
 *     unchanged.
 *   - attn_cached_attention replaces the static cached_attention of
 *     transformer.c:203-248 (one query token against cache rows 0..pos).
 *   - the *_ex entry points take explicit shapes, a stream and a workspace
 *     and return a status instead of exiting.
 *
 * Everything here is plain C: pointers, sizes, ints.  All tensor pointers are
 * DEVICE pointers unless a comment says otherwise.  A stream argument of NULL
 * means the legacy default stream, as the reference uses.
 *
 * Layout (transformer.h:15-18): an activation is a row-major matrix with one
 * row per token; head h of a token occupies columns [h*d, (h+1)*d).  Rows are
 * `row_stride` elements apart (heads*head_dim for a dense tensor, D_MODEL in
 * the reference).  Token t of batch b is row b*T + t.
 */
#ifndef ATTN_B200_H
#define ATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ATTN_API __attribute__((visibility("default")))
#else
#define ATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *attn_stream_t;   /* a cudaStream_t */

/* status codes returned by every int-returning entry point */
enum {
    ATTN_OK = 0,
    ATTN_ERR_INVALID = 1,      /* bad pointer, shape, stride or alignment      */
    ATTN_ERR_UNSUPPORTED = 2,  /* valid request this build has no kernel for   */
    ATTN_ERR_CUDA = 3,         /* a CUDA runtime/driver call failed            */
    ATTN_ERR_NOMEM = 4,        /* device allocation failed                     */
    ATTN_ERR_WORKSPACE = 5,    /* caller workspace smaller than required       */
    ATTN_ERR_DEVICE = 6,       /* a kernel reported an internal error (bounded
                                  wait expired); see attn_device_error()       */
    ATTN_ERR_COMM = 7          /* a collective failed or a group wait timed
                                  out; the group has been torn down           */
};

/* element types of activations / caches */
enum {
    ATTN_F32 = 0,    /* float32 storage, float32 arithmetic (the reference's)  */
    ATTN_BF16 = 1,   /* bf16 storage, bf16 tensor-core products, fp32 accumulate */
    ATTN_I8 = 2      /* int8 KV cache codes + per-(token, head) fp32 scale      */
};

/* ------------------------------------------------------------------------
 * Errors
 * ---------------------------------------------------------------------- */
/* Text of the last failure on the calling host thread ("" if none). */
ATTN_API const char *attn_last_error(void);
/* Reads and clears the device-side error word of `device` (0 = none).  Bounded
 * waits inside kernels record a code here instead of hanging. */
ATTN_API int attn_device_error(int device, int *code_out);
/* Library version, (major << 16) | minor. */
ATTN_API int attn_version(void);

/* ------------------------------------------------------------------------
 * Training attention, drop-in (gpu_kernels.h:66-72)
 * ---------------------------------------------------------------------- */
/* A C++ translation unit that also includes the reference's gpu_kernels.h
 * (which declares attn_fwd / attn_bwd with C++ linkage) defines
 * ATTN_OMIT_MACRO_DROPINS before including this header, so the two
 * declarations do not conflict; the library exports both linkages. */
#ifndef ATTN_OMIT_MACRO_DROPINS
/* Replaces gpu_kernels.h:67 attn_fwd.  Q,K,V,att: (B*T, H*d) fp32 device.
 * `probs` is the caller's buffer (B*H*T*T floats in train_kaggle.cu:123,128).
 * In the default mode (ATTN_PROBS_LSE_OUT) this library stores the per-row
 * log-sum-exp and a copy of the output there, which attn_bwd reads back:
 * probs needs B*H*T*(1+d) floats, and T >= d+1.  In ATTN_PROBS_LSE mode it
 * stores only the log-sum-exp (B*H*T floats, any T) and attn_bwd reads the
 * output from `att` itself (see attn_set_probs_mode).  Sets att.  Exits(1)
 * with a message on failure. */
ATTN_API void attn_fwd(const float *Q, const float *K, const float *V, float *att, float *probs);

/* Replaces gpu_kernels.h:70 attn_bwd.  SETS dQ, dK, dV (like the reference's
 * cuBLAS path, beta = 0).  `scratch` is the caller's workspace (B*H*T*T
 * floats in train_kaggle.cu:138).  At head_dim 96 and 128 with T a multiple
 * of 4 the backward runs as tensor-core GEMMs over explicit score tiles: in
 * the default ATTN_PROBS_LSE_OUT mode this library fills all of `scratch`
 * with dS (as the reference's own softmax backward does) and keeps the
 * scores, P^T, dS^T, the row statistics and split operands in a library-owned
 * device buffer (2*B*H*T*(T+5d+1) floats, 654 MB at the trainer's shape); in
 * ATTN_PROBS_LSE mode dS goes to that buffer as well (B*H*T*T floats more,
 * one buffer for every layer).  Calls that use the buffer must not overlap on
 * the GPU.  Otherwise, or when the buffer cannot be allocated, it runs the
 * CUDA-core kernels and uses 2*B*H*T floats of `scratch`.  Exits(1) with a
 * message on failure. */
ATTN_API void attn_bwd(float *dQ, float *dK, float *dV, float *scratch,
              const float *dAtt, const float *Q, const float *K, const float *V,
              const float *probs);
#endif

/* Shape used by attn_fwd/attn_bwd.  Defaults are gpu_kernels.h:17-31:
 * B_SIZE 4, N_HEADS 12, T_SIZE 1024, D_HEAD 128 (DIM 1536); a build may
 * override them with -DATTN_B_SIZE= etc.  Returns ATTN_OK or an error
 * (ATTN_ERR_UNSUPPORTED for T < d+1 in ATTN_PROBS_LSE_OUT mode). */
ATTN_API int attn_set_macro_shape(int batch, int heads, int seq_len, int head_dim);

/* What attn_fwd keeps in `probs` for attn_bwd.
 *   ATTN_PROBS_LSE_OUT (default): log-sum-exp and a copy of the output,
 *     B*H*T*(1+d) floats; attn_bwd needs nothing else.
 *   ATTN_PROBS_LSE: log-sum-exp only, B*H*T floats -- the trainer's a_probs
 *     shrinks from B*H*T*T floats per layer (2.4 GB at the 343M shape) to
 *     B*H*T, and T is no longer bounded by that allocation.  attn_fwd records
 *     which `att` buffer it wrote for each `probs` buffer; attn_bwd reads the
 *     output from that `att`, which the caller must leave unchanged between
 *     the two calls (train_kaggle.cu keeps a_att[l] for the Wo gradient).
 *     attn_bwd with a `probs` that no attn_fwd of this process has filled is
 *     an error (exit(1), like any drop-in failure).
 * Returns ATTN_OK, or ATTN_ERR_INVALID for another value. */
enum { ATTN_PROBS_LSE_OUT = 0, ATTN_PROBS_LSE = 1 };
ATTN_API int attn_set_probs_mode(int mode);

/* ------------------------------------------------------------------------
 * Training attention, explicit shapes
 * ---------------------------------------------------------------------- */
typedef struct {
    int batch;                  /* B                                          */
    int heads;                  /* H (heads handled by this call)             */
    int seq_len;                /* T                                          */
    int head_dim;               /* d: 32, 64, 96 or 128                       */
    long long in_row_stride;    /* elements between rows of Q,K,V,dO (0: H*d) */
    long long out_row_stride;   /* elements between rows of O,dQ,dK,dV (0: H*d) */
} attn_shape;

/* Causal forward O = softmax(Q K^T / sqrt(d)) V per (b, h), rows j <= i.
 * dtype ATTN_F32: fp32 in/out, fp32 arithmetic (train.c:339-370 semantics).
 * dtype ATTN_BF16: bf16 in/out, tensor-core products, fp32 softmax.  At head
 * dims 32, 96 and 128 a bf16 call keeps fp32 copies of its tensors (4*B*T*H*d
 * floats) in a library-owned device buffer, grown on demand; such calls must
 * not overlap on the GPU.
 * lse (may be NULL): B*H*T floats, [b][h][t] = max + log(sum) of the scaled
 * scores of row t -- the statistic the backward recomputes P from. */
ATTN_API int attn_fwd_ex(const attn_shape *s, int dtype,
                const void *Q, const void *K, const void *V, void *O,
                float *lse, attn_stream_t stream);

/* Bytes of device workspace attn_bwd_ex needs for this shape. */
ATTN_API size_t attn_bwd_workspace_bytes(const attn_shape *s, int dtype);

/* Bytes of workspace that let attn_bwd_ex run an fp32 backward at head_dim 96
 * or 128 (T a multiple of 4, accumulate = 0) on the tensor cores, as GEMMs
 * over explicit score tiles: 2*B*H*T*(T+5d+1) + B*H*T*T floats (the scores,
 * P^T, dS^T, dS, split operands and row statistics; 855 MB at B4 H12 T1024
 * d128), rounded to 256-byte pieces.  0 for shapes without that path.  A
 * smaller workspace (at least attn_bwd_workspace_bytes) selects the CUDA-core
 * kernels. */
ATTN_API size_t attn_bwd_tc_workspace_bytes(const attn_shape *s);

/* Analytic backward (train.c:373-407): dQ, dK, dV from dO, the forward's
 * inputs, its output O and its lse.  accumulate = 1 adds into dQ/dK/dV as
 * train.c does; 0 overwrites them as gpu_kernels.cu's attn_bwd does. */
ATTN_API int attn_bwd_ex(const attn_shape *s, int dtype,
                const void *dO, const void *Q, const void *K, const void *V,
                const void *O, const float *lse,
                void *dQ, void *dK, void *dV, int accumulate,
                void *workspace, size_t workspace_bytes, attn_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused QKV projection (train_kaggle.cu:152-154)
 * ---------------------------------------------------------------------- */
typedef struct {
    int rows;                   /* M: token rows of X (B*T)                    */
    int in_features;            /* columns of X = rows of each W (DIM)         */
    int out_features;           /* N: columns of each W and of each output;
                                   a multiple of 4                              */
    long long x_row_stride;     /* elements between rows of X (0: in_features) */
    long long out_row_stride;   /* elements between rows of Q, K, V
                                   (0: out_features; 3*N for the three column
                                   blocks of one (M, 3N) tensor)                */
} attn_qkv_shape;

/* Bytes of device workspace attn_qkv_proj_ex uses for this shape: the three
 * weights transposed and split, 2 * 3 * out_features * in_features floats
 * (in_features rounded up to 4). */
ATTN_API size_t attn_qkv_workspace_bytes(const attn_qkv_shape *s);

/* Q = X Wq + bq, K = X Wk + bk, V = X Wv + bv: the three gemm_nn calls of
 * train_kaggle.cu:152-154 (gemm_nn: gpu_kernels.cu:112-120, row-major fp32,
 * bias broadcast over rows) in one tensor-core launch, after one small launch
 * that splits the weights.  X (rows, in_features), each W (in_features,
 * out_features) row-major, fp32; biases may be NULL.  fp32 arithmetic (three
 * tf32 products per product, fp32 sums; results within ~1e-6 of an fp32
 * GEMM).  Outputs are SET.  Tensors 16-byte aligned.  `workspace` (256-byte
 * aligned, attn_qkv_workspace_bytes) may be NULL: the library then uses its
 * own per-device buffer, grown on demand, and calls that use it must not
 * overlap on the GPU.  Returns ATTN_OK or a status. */
ATTN_API int attn_qkv_proj_ex(const attn_qkv_shape *s, const float *x,
                const float *wq, const float *wk, const float *wv,
                const float *bq, const float *bk, const float *bv,
                float *q, float *k, float *v,
                void *workspace, size_t workspace_bytes, attn_stream_t stream);

/* The same with gemm_nn's argument style (A, B, bias, C, M, K, N): dense
 * (M, K) input, (K, N) weights, (M, N) outputs, the legacy default stream,
 * void return and exit(1) with a message on failure, like the drop-ins.
 * Replaces train_kaggle.cu:152-154's three calls with one. */
ATTN_API void attn_qkv_proj(const float *X, const float *Wq, const float *Wk, const float *Wv,
                const float *bq, const float *bk, const float *bv,
                float *Q, float *K, float *V, int M, int K_, int N);

/* ------------------------------------------------------------------------
 * KV-cached decode (transformer.c:203-248, model.h:42-45)
 * ---------------------------------------------------------------------- */
typedef struct {
    int n_seq;                  /* independent sequences (or layers) per call */
    int heads;                  /* H                                          */
    int head_dim;               /* d: 32, 64, 96 or 128                       */
    int kv_dtype;               /* ATTN_F32 or ATTN_I8                        */
    long long row_stride;       /* elements between cache rows (0: H*d)      */
    long long cap;              /* rows allocated per sequence's cache        */
    int max_len;                /* upper bound of lens[] (<= cap)             */
} attn_decode_shape;

/* Bytes of device workspace attn_decode_ex / attn_decode_ptrs_ex need. */
ATTN_API size_t attn_decode_workspace_bytes(const attn_decode_shape *s);

/* Decode one query token per sequence against that sequence's cache rows
 * 0..lens[s]-1 (lens[s] = pos+1 in transformer.c terms; lens is a DEVICE
 * int array, each in [1, max_len]; NULL means every sequence attends max_len
 * rows).
 *   q, out: n_seq x (H*d) fp32, dense.
 *   kcache/vcache: sequence s row r at base + (s*cap + r)*row_stride, fp32
 *     (ATTN_F32) or int8 codes (ATTN_I8).
 *   kscale/vscale: ATTN_I8 only, fp32 [(s*cap + r)*H + h] (NULL for fp32).
 * workspace may be NULL: the library then uses a buffer of its own per
 * device (allocated on first use); calls that use that buffer must not
 * overlap on the GPU (order them on one stream, or give each stream its own
 * workspace). */
ATTN_API int attn_decode_ex(const attn_decode_shape *s, const float *q,
                   const void *kcache, const void *vcache,
                   const float *kscale, const float *vscale,
                   const int *lens, float *out,
                   void *workspace, size_t workspace_bytes, attn_stream_t stream);

/* Same, with one cache slab per sequence: kptrs/vptrs (and kscales/vscales
 * for ATTN_I8) are DEVICE arrays of n_seq device pointers, each slab laid out
 * as cap rows of row_stride elements -- the per-layer KVCache.k[l] slabs of
 * model.h:42-45. */
ATTN_API int attn_decode_ptrs_ex(const attn_decode_shape *s, const float *q,
                        const void *const *kptrs, const void *const *vptrs,
                        const float *const *kscales, const float *const *vscales,
                        const int *lens, float *out,
                        void *workspace, size_t workspace_bytes, attn_stream_t stream);

/* No counterpart in the reference.  Same as attn_decode_ex, but it allocates
 * nothing and takes no workspace: the scratch is a fixed array of
 * ATTN_DECODE_STATIC_SCRATCH_BYTES inside the library's device image, reserved
 * on every GPU that loads the library until the process exits.  It is for
 * callers that cannot allocate device memory (memory owned by another
 * allocator, or a loop that must not let cudaMalloc synchronise the device).
 * Shapes whose scratch need (attn_decode_workspace_bytes) exceeds the array
 * are rejected with ATTN_ERR_WORKSPACE.  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress); make that first call
 * before any stream capture.  All calls share the array: calls whose kernels
 * overlap on the GPU race. */
#define ATTN_DECODE_STATIC_SCRATCH_BYTES (4u << 20)
ATTN_API int attn_decode_static_ex(const attn_decode_shape *s, const float *q,
                                   const void *kcache, const void *vcache,
                                   const float *kscale, const float *vscale,
                                   const int *lens, float *out, attn_stream_t stream);

/* cached_attention (transformer.c:203) with device pointers: one token of one
 * layer, attends rows 0..pos.  Writes out (H*d).  Uses the library's own
 * workspace, so calls must not overlap on the GPU with other calls that use
 * it.  Returns a status. */
ATTN_API int attn_cached_attention(const float *q, const float *kcache, const float *vcache,
                          float *out, int pos, int heads, int head_dim,
                          long long row_stride, attn_stream_t stream);

/* cached_attention (transformer.c:203-248) with its own argument list and
 * HOST pointers: a drop-in for the call at transformer.c:266 (forward_block).
 * q, out: H*d floats; kcache/vcache: the caller's host cache, T_MAX rows of
 * H*d floats (transformer.h:35-38 shapes, or attn_set_decode_macro_shape);
 * `scores` is accepted and unused.  The library keeps a device mirror of each
 * (kcache, vcache) pair and copies over only the rows it has not seen -- the
 * generator writes row `pos` before attending (transformer.c:256-264) -- then
 * decodes on the GPU and writes `out` before returning.  A call with a pos
 * below the mirrored length re-sends rows from pos on; rows below pos must not
 * change once sent.  Exits(1) with a message on failure. */
ATTN_API void attn_cached_attention_host(const float *q, const float *kcache, const float *vcache,
                                         float *out, float *scores, int pos);
/* Shapes of attn_cached_attention_host (defaults: transformer.h:35-38,
 * N_HEADS 16, D_HEAD 96, T_MAX 512; rows of heads*head_dim floats). */
ATTN_API int attn_set_decode_macro_shape(int heads, int head_dim, int t_max);
/* The same with explicit shapes and a status (generate.c:130-152 works with
 * run-time dims: H, DH, row stride D, BLK rows). */
ATTN_API int attn_cached_attention_host_ex(const float *q, const float *kcache, const float *vcache,
                                           float *out, int pos, int heads, int head_dim,
                                           long long row_stride, int cap);
/* Frees the device mirror of a host cache pair. */
ATTN_API int attn_host_cache_release(const float *kcache, const float *vcache);

/* INT8 quantiser for caches: the reference's symmetric absmax scheme
 * (gemm_bench.c:225-236: amax floored at 1e-8, scale = amax/127,
 * q = lroundf(x/scale) clamped to +-127) applied per (row, head).
 * x: rows x row_stride fp32; codes: same layout int8; scales: rows x heads. */
ATTN_API int attn_kv_quantize_int8(const float *x, long long rows, int heads, int head_dim,
                          long long row_stride, int8_t *codes, float *scales,
                          attn_stream_t stream);

/* ------------------------------------------------------------------------
 * Device KV cache (model.h:42-48, alloc_kv_cache at model.c:27-33 mallocs
 * host slabs; this one owns device slabs)
 * ---------------------------------------------------------------------- */
#define ATTN_MAX_LAYERS 64
typedef struct {
    int n_layers, cap, heads, head_dim, kv_dtype;
    void *k[ATTN_MAX_LAYERS];        /* cap x (heads*head_dim) per layer      */
    void *v[ATTN_MAX_LAYERS];
    float *kscale[ATTN_MAX_LAYERS];  /* cap x heads per layer (ATTN_I8 only)  */
    float *vscale[ATTN_MAX_LAYERS];
} attn_kv_cache;

ATTN_API int attn_kv_cache_alloc(attn_kv_cache *c, int n_layers, int cap, int heads,
                        int head_dim, int kv_dtype);
ATTN_API int attn_kv_cache_free(attn_kv_cache *c);
/* Writes one token's K and V rows (fp32, H*d each, device) at row `pos` of
 * `layer`, quantising on append for an ATTN_I8 cache -- the row write of
 * transformer.c:260-264. */
ATTN_API int attn_kv_cache_append(attn_kv_cache *c, int layer, int pos,
                         const float *krow, const float *vrow, attn_stream_t stream);

/* ------------------------------------------------------------------------
 * Multi-GPU partitioning by (batch x head) units
 * ---------------------------------------------------------------------- */
/* Contiguous split of n_units over `world` ranks: rank gets [*begin, *end). */
ATTN_API int attn_shard_range(long long n_units, int world, int rank,
                     long long *begin, long long *end);
/* Longest-processing-time-first assignment of (seq, head) decode units whose
 * cost is the cache length: out_rank[s*heads + h] receives the rank,
 * out_load[r] (may be NULL) the summed length per rank.  Host arrays. */
ATTN_API int attn_shard_lpt(const int *lens, int n_seq, int heads, int world,
                   int *out_rank, long long *out_load);
/* After an all-gather of head shards, staging is [world][B][T][H/world][d];
 * writes out as (B*T, H*d).  dtype ATTN_F32 or ATTN_BF16. */
ATTN_API int attn_gather_permute(const void *staging, void *out, int world, int batch,
                        int seq_len, int heads, int head_dim, int dtype,
                        attn_stream_t stream);

/* ------------------------------------------------------------------------
 * Multi-GPU groups (no counterpart in the reference, whose trainer drives one
 * GPU from one host process, train_kaggle.cu:346).  NCCL over NVLink is used
 * only to gather outputs for callers that need them whole; the attention
 * itself needs no collective.  NCCL is loaded at run time (libnccl.so.2, or
 * the path in $ATTN_NCCL_LIB); NCCL_NVLS_ENABLE defaults to 0.  One group per
 * process.
 * ---------------------------------------------------------------------- */
/* One host thread drives devices 0..ngpus-1 (ncclCommInitAll); use
 * attn_fwd_multi / attn_decode_multi. */
ATTN_API int attn_init(int ngpus);
/* One process per GPU: rank 0 makes a 128-byte id, the caller hands it to
 * every rank, and each joins with attn_init_rank on `device` (-1: the current
 * device); then use the ordinary entry points on the rank's share and
 * attn_gather_split / attn_gather_rows. */
ATTN_API int attn_get_unique_id(unsigned char id[128]);
ATTN_API int attn_init_rank(int nranks, int rank, int device, const unsigned char id[128]);
/* Destroys the group's communicators (after the caller's work on them is done). */
ATTN_API int attn_finalize(void);
/* Ranks in the group, 0 when there is none. */
ATTN_API int attn_group_size(void);
/* Host-side watchdog: waits until every listed stream is idle, polling the
 * communicators' asynchronous errors.  On a communicator error, or when the
 * streams are still busy after timeout_ms, it aborts every communicator
 * (ncclCommAbort), removes the group and returns ATTN_ERR_COMM. */
ATTN_API int attn_group_sync(const attn_stream_t *streams, int n_streams, int timeout_ms);

/* A rank's share of the (batch x head) units: nb x nh ranks tile the batch and
 * head ranges evenly, with as many ranks along the batch as divide it (whole
 * batches keep a rank's rows contiguous).  Rank r holds batches
 * [batch0, batch0 + batch) and heads [head0, head0 + heads). */
typedef struct {
    int batch0, batch, head0, heads;
    int nb, nh;
} attn_split;
ATTN_API int attn_split_plan(int batch, int heads, int nranks, int rank, attn_split *out);

/* Bytes of workspace attn_gather_split / attn_fwd_multi need per rank for a
 * gather of this shape (0 when the split is by whole batches). */
ATTN_API size_t attn_gather_workspace_bytes(const attn_shape *s, int dtype, int nranks);
/* One-process-per-rank group: `local` is this rank's forward output, dense
 * (batch*T rows of heads*d, its split of `s`, the full shape); writes the
 * whole (B*T, H*d) output `out` on every rank (all-gather, then a permute
 * kernel when ranks split the heads). */
ATTN_API int attn_gather_split(const attn_shape *s, int dtype, const void *local, void *out,
                               void *workspace, size_t workspace_bytes, attn_stream_t stream);

/* Ragged decode across ranks: each rank decodes its own sequences (for
 * example by attn_shard_lpt with heads = 1) into `local`, max_local rows of
 * row_bytes (a multiple of 16).  attn_gather_rows all-gathers every rank's
 * max_local rows and writes row i of the gathered [nranks][max_local] block to
 * out row order[i] (a DEVICE array; < 0 skips padding).  order == NULL: the
 * gathered block is the output (n_out = nranks * max_local). */
ATTN_API size_t attn_gather_rows_workspace_bytes(int max_local, size_t row_bytes, int nranks);
ATTN_API int attn_gather_rows(const void *local, int max_local, size_t row_bytes, const int *order,
                              int n_out, void *out, void *workspace, size_t workspace_bytes,
                              attn_stream_t stream);

/* attn_init group, one host thread: device g holds the full-size inputs
 * q[g], k[g], v[g] (shape `s`) and runs its split (attn_split_plan with
 * rank g) into o[g] at the split's rows and columns; lse[g] (may be NULL)
 * receives its split's [batch][heads][T] statistics.  gather = 1 completes
 * o[g] on every device (NCCL all-gather on streams[g]; dense output rows
 * needed); ws[g] / ws_bytes[g] as attn_gather_workspace_bytes. */
ATTN_API int attn_fwd_multi(const attn_shape *s, int dtype, const void *const *q,
                            const void *const *k, const void *const *v, void *const *o,
                            float *const *lse, int gather, void *const *ws,
                            const size_t *ws_bytes, const attn_stream_t *streams);
/* attn_init group, one host thread: device g decodes its own sequences
 * (shapes[g], its caches and lens, out[g] with max_local rows); gather = 1
 * then writes every device's rows into out_full[g] (n_total rows, 16-byte
 * aligned) by order[g] (as attn_gather_rows), with ws[g] of
 * attn_gather_rows_workspace_bytes(max_local, H*d*4, ngpus) bytes. */
ATTN_API int attn_decode_multi(const attn_decode_shape *shapes, const float *const *q,
                               const void *const *kcache, const void *const *vcache,
                               const float *const *kscale, const float *const *vscale,
                               const int *const *lens, float *const *out, int gather,
                               int max_local, const int *const *order, int n_total,
                               float *const *out_full, void *const *ws,
                               const size_t *ws_bytes, const attn_stream_t *streams);

/* ------------------------------------------------------------------------
 * Test hook (no counterpart in the reference)
 * ---------------------------------------------------------------------- */
/* The next `launches` fp32 decode calls served by the TMA-ring decode kernel
 * (fp32 calls of up to 256 sequences and 256 MB of cache that are too large
 * for the one-CTA-per-head kernel) make one of its warps wait on a
 * barrier that nothing arrives at, bounded by `limit_cycles` SM cycles
 * (>= 1000).  The wait runs out and the kernel takes its timeout path: it
 * records code 0x32f in the device error word (attn_device_error), stops,
 * lets the copies it has in flight land, and returns; the call's output is
 * undefined and later calls run normally.  For tests of failure detection:
 * no GPU fault is involved. */
ATTN_API int attn_debug_decode_timeout(int launches, long long limit_cycles);

/* The same for the next `launches` calls of the QKV projection: the MMA
 * warp of its tensor-core kernel first waits on a barrier that nothing
 * arrives at, bounded by `limit_cycles` (>= 1000).  The kernel records 0x5ff
 * in the device error word, every role stops, and the teardown frees the
 * kernel's TMEM; the call's outputs are undefined and later calls run
 * normally. */
ATTN_API int attn_debug_qkv_timeout(int launches, long long limit_cycles);

#ifdef __cplusplus
}
#endif

#endif /* ATTN_B200_H */
