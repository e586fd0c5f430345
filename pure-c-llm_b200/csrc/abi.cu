// abi.cu -- the C ABI of libattn_b200 (include/attn_b200.h): argument
// checking, workspaces, the macro-shaped drop-ins for gpu_kernels.h, the device
// KV cache, and the multi-GPU partition helpers.
#include "decode_launch.cuh"
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <tuple>
#include <unordered_map>
#include <mutex>
#include <queue>
#include <utility>
#include <vector>

#include "common.cuh"

#ifndef ATTN_B_SIZE
#define ATTN_B_SIZE 4       /* gpu_kernels.h:29 */
#endif
#ifndef ATTN_N_HEADS
#define ATTN_N_HEADS 12     /* gpu_kernels.h:19 */
#endif
#ifndef ATTN_T_SIZE
#define ATTN_T_SIZE 1024    /* gpu_kernels.h:22,31 */
#endif
#ifndef ATTN_D_HEAD
#define ATTN_D_HEAD 128     /* gpu_kernels.h:20 (1536 / 12) */
#endif

// ---- kernels' host launchers (other translation units) ----------------------
namespace attn_host {
int launch_decode(const DecodeLaunch &L);
size_t decode_workspace_bytes(int n_seq, int heads, int head_dim, int max_len, int kv_dtype);
int launch_fwd_f32(int dtype, int D, const void *q, const void *k, const void *v, void *o,
                   float *lse, long long in_stride, long long out_stride, int B, int H, int T,
                   cudaStream_t s);
int launch_fwd_bf16_sm100(int D, const void *q, const void *k, const void *v, void *o, float *lse,
                          long long in_stride, long long out_stride, int B, int H, int T,
                          int *err, cudaStream_t s);
bool fwd_bf16_sm100_supported(int D, long long in_stride, long long out_stride);
int launch_fwd_tf32_sm100(int D, const void *q, const void *k, const void *v, void *o, float *lse,
                          long long in_stride, long long out_stride, int B, int H, int T, int *err,
                          cudaStream_t s, int parts);
int launch_fwd_bf16_via_tf32(int D, const void *q, const void *k, const void *v, void *o, float *lse,
                             long long in_stride, long long out_stride, int B, int H, int T, int *err,
                             cudaStream_t s);
bool fwd_tf32_sm100_supported(int D, long long in_stride, long long out_stride);
int launch_bwd_f32(int dtype, int D, const void *dout, const void *q, const void *k,
                   const void *v, const void *o, const float *lse, void *dq, void *dk, void *dv,
                   int accumulate, void *ws, long long in_stride, long long out_stride, int B,
                   int H, int T, cudaStream_t s);
size_t bwd_f32_workspace_bytes(int B, int H, int T);
size_t bwd_tc_ws_bytes(int B, int H, int T, int D);
int launch_bwd_tc(int D, const float *dout, const float *q, const float *k, const float *v, const float *o,
                  const float *lse, float *dq, float *dk, float *dv, float *ds, void *ws, long long in_stride,
                  long long out_stride, int B, int H, int T, int *err, cudaStream_t s);
void *library_workspace(int which, size_t bytes, cudaStream_t s);
bool bwd_bf16_sm100_supported(int D, long long in_stride, long long out_stride);
bool bwd_tf32_sm100_supported(int D, long long in_stride, long long out_stride);
int launch_bwd_tf32_sm100(int D, const void *dout, const void *q, const void *k, const void *v, const void *o,
                          const float *lse, void *dq, void *dk, void *dv, int accumulate, void *ws,
                          long long in_stride, long long out_stride, int B, int H, int T, int *err,
                          cudaStream_t s);
int launch_bwd_bf16_sm100(int D, const void *dout, const void *q, const void *k, const void *v, const void *o,
                          const float *lse, void *dq, void *dk, void *dv, int accumulate, void *ws,
                          long long in_stride, long long out_stride, int B, int H, int T, int *err,
                          cudaStream_t s);
int launch_quantize_int8(const float *x, long long rows, int heads, int head_dim,
                         long long row_stride, int8_t *codes, float *scales, cudaStream_t s);
int launch_append_f32(const float *krow, const float *vrow, float *kdst, float *vdst, int n,
                      cudaStream_t s);
int launch_gather_permute(const void *staging, void *out, int G, int B, int T, int H, int D,
                          int dtype, cudaStream_t s);
}  // namespace attn_host

// Device-side error word, one per device (module-scope variable).  Kernels with
// bounded waits write a nonzero code here instead of hanging.
__device__ int g_attn_device_error;

namespace attn_host {

static thread_local char g_err[512];

int set_error(int status, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
    return status;
}

static std::mutex g_mu;

bool ensure_smem_attr(const void *func, size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    static std::map<std::pair<const void *, int>, size_t> done;
    std::lock_guard<std::mutex> lk(g_mu);
    auto key = std::make_pair(func, dev);
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return true;
    if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
        return false;
    done[key] = bytes;
    return true;
}

// Per-device cache of the persistent kernels' schedules (per-CTA item lists),
// one immutable device buffer per (kernel, shape) key.  A buffer is written
// once, synchronously on a private stream, before its first use and never
// again, so calls of different shapes may overlap on any streams.  The first
// call of a new shape allocates and uploads (keep it out of stream capture).
// After kMaxSchedules shapes on a device, the callers fall back to their
// list-free static schedule.
const unsigned short *schedule_get(int kernel_tag, long long key,
                                   const std::function<void(std::vector<unsigned short> &)> &build) {
    constexpr size_t kMaxSchedules = 256;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    static std::map<std::tuple<int, int, long long>, unsigned short *> cache;
    static std::map<int, cudaStream_t> upload_stream;
    std::lock_guard<std::mutex> lk(g_mu);
    const auto k = std::make_tuple(dev, kernel_tag, key);
    auto it = cache.find(k);
    if (it != cache.end()) return it->second;
    if (cache.size() >= kMaxSchedules * 8) return nullptr;
    size_t on_dev = 0;
    for (auto &e : cache) on_dev += std::get<0>(e.first) == dev;
    if (on_dev >= kMaxSchedules) return nullptr;
    std::vector<unsigned short> h;
    build(h);
    cudaStream_t &us = upload_stream[dev];
    if (!us && cudaStreamCreateWithFlags(&us, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    unsigned short *d = nullptr;
    if (cudaMalloc(&d, h.size() * sizeof(unsigned short)) != cudaSuccess) return nullptr;
    if (cudaMemcpyAsync(d, h.data(), h.size() * sizeof(unsigned short), cudaMemcpyHostToDevice, us) != cudaSuccess ||
        cudaStreamSynchronize(us) != cudaSuccess) {
        cudaFree(d);
        return nullptr;
    }
    cache[k] = d;
    return d;
}

// SM count of the current device, cached.
int sm_count_here() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    static std::map<int, int> counts;
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = counts.find(dev);
    if (it != counts.end()) return it->second;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = sms;
    return sms;
}

// Sets a kernel's preferred shared-memory carveout once per device.
bool ensure_carveout(const void *func, int percent) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    static std::map<std::pair<const void *, int>, int> done;
    std::lock_guard<std::mutex> lk(g_mu);
    auto key = std::make_pair(func, dev);
    if (done.count(key)) return true;
    if (cudaFuncSetAttribute(func, cudaFuncAttributePreferredSharedMemoryCarveout, percent) != cudaSuccess)
        return false;
    done[key] = percent;
    return true;
}

int *device_error_ptr() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    static std::map<int, int *> ptrs;
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = ptrs.find(dev);
    if (it != ptrs.end()) return it->second;
    int *p = nullptr;
    if (cudaGetSymbolAddress((void **)&p, g_attn_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = p;
    return p;
}

// Library-owned decode workspace, one per device, grown on demand.  Its
// ticket words start at zero (memset at allocation) and every decode call
// leaves them at zero.  Calls that share it must be ordered on one stream.
static void *internal_workspace(size_t bytes, cudaStream_t s) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    static std::map<int, std::pair<void *, size_t>> pool;
    std::lock_guard<std::mutex> lk(g_mu);
    auto &slot = pool[dev];
    if (slot.second >= bytes) return slot.first;
    if (slot.first) {
        cudaStreamSynchronize(s);
        cudaFree(slot.first);
        slot = {nullptr, 0};
    }
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, bytes) != cudaSuccess) { cudaFree(p); return nullptr; }
    slot = {p, bytes};
    return p;
}

static bool aligned(const void *p, size_t a) { return ((uintptr_t)p % a) == 0; }
static bool head_dim_ok(int d) { return d == 32 || d == 64 || d == 96 || d == 128; }

}  // namespace attn_host

using namespace attn_host;

// ===========================================================================
extern "C" {

const char *attn_last_error(void) { return g_err; }

int attn_version(void) { return (0 << 16) | 1; }

int attn_device_error(int device, int *code_out) {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return set_error(ATTN_ERR_CUDA, "cudaGetDevice failed");
    if (cudaSetDevice(device) != cudaSuccess) return set_error(ATTN_ERR_INVALID, "bad device %d", device);
    int code = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&code, g_attn_device_error, sizeof(int));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_attn_device_error, &zero, sizeof(int));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(ATTN_ERR_CUDA, "device error word: %s", cudaGetErrorString(e));
    if (code_out) *code_out = code;
    return ATTN_OK;
}

// ---------------------------------------------------------------------------
// training attention
// ---------------------------------------------------------------------------
static int check_shape(const attn_shape *s, int dtype, long long *in_st, long long *out_st) {
    if (!s) return set_error(ATTN_ERR_INVALID, "shape is NULL");
    if (s->batch < 0 || s->heads < 1 || s->seq_len < 0)
        return set_error(ATTN_ERR_INVALID, "bad shape B=%d H=%d T=%d", s->batch, s->heads, s->seq_len);
    if (!head_dim_ok(s->head_dim))
        return set_error(ATTN_ERR_UNSUPPORTED, "head_dim %d not in {32,64,96,128}", s->head_dim);
    if (dtype != ATTN_F32 && dtype != ATTN_BF16)
        return set_error(ATTN_ERR_UNSUPPORTED, "dtype %d not supported for training attention", dtype);
    const long long hd = (long long)s->heads * s->head_dim;
    *in_st = s->in_row_stride ? s->in_row_stride : hd;
    *out_st = s->out_row_stride ? s->out_row_stride : hd;
    if (*in_st < hd || *out_st < hd || (*in_st % 4) || (*out_st % 4))
        return set_error(ATTN_ERR_INVALID, "row strides (%lld, %lld) must be >= H*d=%lld and multiples of 4",
                         *in_st, *out_st, hd);
    return ATTN_OK;
}

int attn_fwd_ex(const attn_shape *s, int dtype, const void *Q, const void *K, const void *V,
                void *O, float *lse, attn_stream_t stream) {
    long long in_st, out_st;
    int st = check_shape(s, dtype, &in_st, &out_st);
    if (st) return st;
    if (s->batch == 0 || s->seq_len == 0) return ATTN_OK;
    const size_t al = dtype == ATTN_F32 ? 16 : 8;
    if (!Q || !K || !V || !O) return set_error(ATTN_ERR_INVALID, "fwd: NULL tensor pointer");
    if (!aligned(Q, al) || !aligned(K, al) || !aligned(V, al) || !aligned(O, al) || (lse && !aligned(lse, 4)))
        return set_error(ATTN_ERR_INVALID, "fwd: tensors must be %zu-byte aligned", al);
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == ATTN_BF16 && fwd_bf16_sm100_supported(s->head_dim, in_st, out_st))
        return launch_fwd_bf16_sm100(s->head_dim, Q, K, V, O, lse, in_st, out_st, s->batch,
                                     s->heads, s->seq_len, device_error_ptr(), cs);
    if (dtype == ATTN_F32 && fwd_tf32_sm100_supported(s->head_dim, in_st, out_st))
        return launch_fwd_tf32_sm100(s->head_dim, Q, K, V, O, lse, in_st, out_st, s->batch,
                                     s->heads, s->seq_len, device_error_ptr(), cs, 3);
    // bf16 at the other head dims: the tf32 kernel over exact fp32 copies, one product per product
    if (dtype == ATTN_BF16 && fwd_tf32_sm100_supported(s->head_dim, s->heads * (long long)s->head_dim,
                                                       s->heads * (long long)s->head_dim) &&
        in_st % 4 == 0 && out_st % 4 == 0) {
        const int st = launch_fwd_bf16_via_tf32(s->head_dim, Q, K, V, O, lse, in_st, out_st, s->batch, s->heads,
                                                s->seq_len, device_error_ptr(), cs);
        if (st != ATTN_ERR_NOMEM) return st;
    }
    return launch_fwd_f32(dtype, s->head_dim, Q, K, V, O, lse, in_st, out_st, s->batch, s->heads,
                          s->seq_len, cs);
}

size_t attn_bwd_workspace_bytes(const attn_shape *s, int dtype) {
    (void)dtype;
    if (!s) return 0;
    return bwd_f32_workspace_bytes(s->batch, s->heads, s->seq_len);
}

size_t attn_bwd_tc_workspace_bytes(const attn_shape *s) {
    if (!s || (s->head_dim != 96 && s->head_dim != 128) || s->batch < 1 || s->heads < 1 || s->seq_len < 1 ||
        s->seq_len % 4 || (long long)s->batch * s->heads > 65535)
        return 0;
    return bwd_tc_ws_bytes(s->batch, s->heads, s->seq_len, s->head_dim) +
           ((size_t)s->batch * s->heads * s->seq_len * s->seq_len * sizeof(float) + 255) / 256 * 256;
}

int attn_bwd_ex(const attn_shape *s, int dtype, const void *dO, const void *Q, const void *K,
                const void *V, const void *O, const float *lse, void *dQ, void *dK, void *dV,
                int accumulate, void *workspace, size_t workspace_bytes, attn_stream_t stream) {
    long long in_st, out_st;
    int st = check_shape(s, dtype, &in_st, &out_st);
    if (st) return st;
    if (s->batch == 0 || s->seq_len == 0) return ATTN_OK;
    if (!dO || !Q || !K || !V || !O || !lse || !dQ || !dK || !dV)
        return set_error(ATTN_ERR_INVALID, "bwd: NULL pointer");
    const size_t al = dtype == ATTN_F32 ? 16 : 8;
    if (!aligned(dO, al) || !aligned(Q, al) || !aligned(K, al) || !aligned(V, al) || !aligned(O, al) ||
        !aligned(dQ, al) || !aligned(dK, al) || !aligned(dV, al))
        return set_error(ATTN_ERR_INVALID, "bwd: tensors must be %zu-byte aligned", al);
    const size_t need = attn_bwd_workspace_bytes(s, dtype);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 16))
        return set_error(ATTN_ERR_WORKSPACE, "bwd: workspace needs %zu bytes (16-byte aligned), got %zu",
                         need, workspace_bytes);
    if (dtype == ATTN_BF16 && bwd_bf16_sm100_supported(s->head_dim, in_st, out_st))
        return launch_bwd_bf16_sm100(s->head_dim, dO, Q, K, V, O, lse, dQ, dK, dV, accumulate ? 1 : 0, workspace,
                                     in_st, out_st, s->batch, s->heads, s->seq_len, device_error_ptr(),
                                     reinterpret_cast<cudaStream_t>(stream));
    if (dtype == ATTN_F32 && bwd_tf32_sm100_supported(s->head_dim, in_st, out_st))
        return launch_bwd_tf32_sm100(s->head_dim, dO, Q, K, V, O, lse, dQ, dK, dV, accumulate ? 1 : 0, workspace,
                                     in_st, out_st, s->batch, s->heads, s->seq_len, device_error_ptr(),
                                     reinterpret_cast<cudaStream_t>(stream));
    // d 96 / 128 with the larger workspace: the tensor-core GEMMs over score tiles
    const size_t tc_need = attn_bwd_tc_workspace_bytes(s);
    if (dtype == ATTN_F32 && !accumulate && tc_need && workspace_bytes >= tc_need && aligned(workspace, 256) &&
        in_st % 4 == 0 && out_st % 4 == 0) {
        const size_t tc = bwd_tc_ws_bytes(s->batch, s->heads, s->seq_len, s->head_dim);
        return launch_bwd_tc(s->head_dim, static_cast<const float *>(dO), static_cast<const float *>(Q),
                             static_cast<const float *>(K), static_cast<const float *>(V),
                             static_cast<const float *>(O), lse, static_cast<float *>(dQ), static_cast<float *>(dK),
                             static_cast<float *>(dV), reinterpret_cast<float *>(static_cast<char *>(workspace) + tc),
                             workspace, in_st, out_st, s->batch, s->heads, s->seq_len, device_error_ptr(),
                             reinterpret_cast<cudaStream_t>(stream));
    }
    return launch_bwd_f32(dtype, s->head_dim, dO, Q, K, V, O, lse, dQ, dK, dV, accumulate ? 1 : 0,
                          workspace, in_st, out_st, s->batch, s->heads, s->seq_len,
                          reinterpret_cast<cudaStream_t>(stream));
}

// ---- macro-shaped drop-ins (gpu_kernels.h:67-72) ---------------------------
}  // extern "C"
namespace attn_host {
void dropin_fwd(const float *Q, const float *K, const float *V, float *att, float *probs);
void dropin_bwd(float *dQ, float *dK, float *dV, float *scratch, const float *dAtt, const float *Q,
                const float *K, const float *V, const float *probs);
}  // namespace attn_host
extern "C" {

static attn_shape g_macro = {ATTN_B_SIZE, ATTN_N_HEADS, ATTN_T_SIZE, ATTN_D_HEAD, 0, 0};
static int g_probs_mode = ATTN_PROBS_LSE_OUT;

int attn_set_macro_shape(int batch, int heads, int seq_len, int head_dim) {
    if (batch < 1 || heads < 1 || seq_len < 1 || !head_dim_ok(head_dim))
        return set_error(ATTN_ERR_INVALID, "bad macro shape B=%d H=%d T=%d d=%d", batch, heads, seq_len, head_dim);
    if (g_probs_mode == ATTN_PROBS_LSE_OUT && seq_len < head_dim + 1)
        return set_error(ATTN_ERR_UNSUPPORTED,
                         "attn_fwd keeps lse + output in `probs`; needs T >= d+1 (T=%d d=%d)", seq_len, head_dim);
    g_macro = {batch, heads, seq_len, head_dim, 0, 0};
    return ATTN_OK;
}

int attn_set_probs_mode(int mode) {
    if (mode != ATTN_PROBS_LSE_OUT && mode != ATTN_PROBS_LSE)
        return set_error(ATTN_ERR_INVALID, "probs mode %d: expected ATTN_PROBS_LSE_OUT or ATTN_PROBS_LSE", mode);
    g_probs_mode = mode;
    return ATTN_OK;
}

// The reference's CUDA_CHECK prints and exits (gpu_kernels.h:34-36); the
// drop-ins keep that behaviour.
static void die_on(int st, const char *where) {
    if (st == ATTN_OK) return;
    fprintf(stderr, "CUDA error '%s' at %s\n", g_err, where);
    exit(1);
}

void attn_fwd(const float *Q, const float *K, const float *V, float *att, float *probs) {
    attn_host::dropin_fwd(Q, K, V, att, probs);
}

void attn_bwd(float *dQ, float *dK, float *dV, float *scratch, const float *dAtt, const float *Q,
              const float *K, const float *V, const float *probs) {
    attn_host::dropin_bwd(dQ, dK, dV, scratch, dAtt, Q, K, V, probs);
}

}  // extern "C"

namespace attn_host {

// Bodies of the drop-ins, shared by the C symbols above and the C++-linkage
// symbols of abi_cxx.cu (train_kaggle.cu and gpu_kernels.h are compiled as
// CUDA C++, so an unchanged trainer references the mangled names).
// ATTN_PROBS_LSE mode: the output buffer each `probs` buffer's forward wrote
// (the backward reads the output from there).  A trainer has one entry per
// layer; the table is bounded so that a caller cycling through fresh buffers
// cannot grow it without end.
static std::mutex g_probs_mu;
static std::unordered_map<const float *, const float *> g_probs_att;
constexpr size_t kProbsEntries = 4096;

void dropin_fwd(const float *Q, const float *K, const float *V, float *att, float *probs) {
    const attn_shape &s = g_macro;
    const bool lse_only = g_probs_mode == ATTN_PROBS_LSE;
    if (!lse_only && s.seq_len < s.head_dim + 1) die_on(set_error(ATTN_ERR_UNSUPPORTED, "T < d+1"), "attn_fwd");
    // probs layout: [lse: B*H*T] then, unless lse_only, [copy of att: B*T*H*d]
    float *lse = probs;
    die_on(attn_fwd_ex(&s, ATTN_F32, Q, K, V, att, lse, nullptr), "attn_fwd");
    if (lse_only) {
        std::lock_guard<std::mutex> g(g_probs_mu);
        if (g_probs_att.size() >= kProbsEntries && !g_probs_att.count(probs)) g_probs_att.clear();
        g_probs_att[probs] = att;
        return;
    }
    float *ocopy = probs + (size_t)s.batch * s.heads * s.seq_len;
    const size_t bytes = (size_t)s.batch * s.seq_len * s.heads * s.head_dim * sizeof(float);
    cudaError_t e = cudaMemcpyAsync(ocopy, att, bytes, cudaMemcpyDeviceToDevice, nullptr);
    if (e != cudaSuccess) die_on(set_error(ATTN_ERR_CUDA, "%s", cudaGetErrorString(e)), "attn_fwd");
}

void dropin_bwd(float *dQ, float *dK, float *dV, float *scratch, const float *dAtt, const float *Q,
                const float *K, const float *V, const float *probs) {
    const attn_shape &s = g_macro;
    const float *lse = probs;
    const float *out = probs + (size_t)s.batch * s.heads * s.seq_len;
    if (g_probs_mode == ATTN_PROBS_LSE) {
        std::lock_guard<std::mutex> g(g_probs_mu);
        auto it = g_probs_att.find(probs);
        if (it == g_probs_att.end())
            die_on(set_error(ATTN_ERR_INVALID, "attn_bwd: no attn_fwd has filled this `probs` buffer "
                                               "(ATTN_PROBS_LSE mode)"), "attn_bwd");
        out = it->second;
    }
    // d 96 and 128 (the fused 3xTF32 backward does not fit TMEM there): in the
    // default probs mode the caller's scratch is the reference's B*H*T*T
    // floats (train_kaggle.cu:138, which its own softmax backward fills with
    // dS), so the backward runs as tensor-core GEMMs over explicit score
    // tiles: dS goes to scratch, the scores, P^T, dS^T, the row statistics and
    // the split operands to a library-owned buffer.
    // In ATTN_PROBS_LSE mode the trainer's scratch is shrunk to 2*B*H*T floats,
    // so dS goes to the library-owned buffer too (one B*H*T*T buffer for all
    // layers, where the reference keeps one per layer).
    const bool lse_mode = g_probs_mode == ATTN_PROBS_LSE;
    if ((s.head_dim == 96 || s.head_dim == 128) && s.seq_len % 4 == 0 &&
        (long long)s.batch * s.heads <= 65535 &&
        ((reinterpret_cast<uintptr_t>(scratch) | reinterpret_cast<uintptr_t>(dQ) | reinterpret_cast<uintptr_t>(dK) |
          reinterpret_cast<uintptr_t>(dV) | reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) |
          reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(dAtt) | reinterpret_cast<uintptr_t>(out)) &
         15) == 0) {
        const long long hd = (long long)s.heads * s.head_dim;
        const size_t tc = bwd_tc_ws_bytes(s.batch, s.heads, s.seq_len, s.head_dim);
        const size_t ds_bytes = lse_mode ? (size_t)s.batch * s.heads * s.seq_len * s.seq_len * sizeof(float) : 0;
        if (void *ws = library_workspace(1, tc + ds_bytes, nullptr)) {
            float *ds = lse_mode ? reinterpret_cast<float *>(static_cast<char *>(ws) + tc) : scratch;
            die_on(launch_bwd_tc(s.head_dim, static_cast<const float *>(dAtt), Q, K, V, static_cast<const float *>(out),
                                 lse, dQ, dK, dV, ds, ws, hd, hd, s.batch, s.heads, s.seq_len, device_error_ptr(),
                                 nullptr),
                   "attn_bwd");
            return;
        }
        (void)cudaGetLastError();      // no room for the buffer: the CUDA-core kernels below need none
    }
    // the caller's scratch holds at least what the backward needs (the
    // reference allocates B*H*T*T floats; a shrunk trainer 2*B*H*T)
    const size_t ws_bytes = attn_bwd_workspace_bytes(&s, ATTN_F32);
    die_on(attn_bwd_ex(&s, ATTN_F32, dAtt, Q, K, V, out, lse, dQ, dK, dV, 0, scratch, ws_bytes, nullptr),
           "attn_bwd");
}

}  // namespace attn_host

extern "C" {

// ---------------------------------------------------------------------------
// decode
// ---------------------------------------------------------------------------
static int check_decode(const attn_decode_shape *s, long long *rs) {
    if (!s) return set_error(ATTN_ERR_INVALID, "decode shape is NULL");
    if (s->n_seq < 0 || s->heads < 1 || s->max_len < 1 || s->n_seq > 65535 || s->heads > 65535)
        return set_error(ATTN_ERR_INVALID, "bad decode shape n_seq=%d H=%d max_len=%d", s->n_seq, s->heads, s->max_len);
    if (!head_dim_ok(s->head_dim))
        return set_error(ATTN_ERR_UNSUPPORTED, "decode: head_dim %d not in {32,64,96,128}", s->head_dim);
    if (s->kv_dtype != ATTN_F32 && s->kv_dtype != ATTN_I8)
        return set_error(ATTN_ERR_UNSUPPORTED, "decode: kv_dtype %d not supported", s->kv_dtype);
    const long long hd = (long long)s->heads * s->head_dim;
    *rs = s->row_stride ? s->row_stride : hd;
    if (*rs < hd || (*rs % (s->kv_dtype == ATTN_F32 ? 4 : 16)))
        return set_error(ATTN_ERR_INVALID, "decode: row_stride %lld must be >= H*d and a multiple of %d",
                         *rs, s->kv_dtype == ATTN_F32 ? 4 : 16);
    if (s->cap < s->max_len) return set_error(ATTN_ERR_INVALID, "decode: cap %lld < max_len %d", s->cap, s->max_len);
    return ATTN_OK;
}

size_t attn_decode_workspace_bytes(const attn_decode_shape *s) {
    if (!s || s->n_seq < 1 || s->heads < 1 || s->max_len < 1) return 0;
    return decode_workspace_bytes(s->n_seq, s->heads, s->head_dim, s->max_len, s->kv_dtype);
}

static int decode_common(const attn_decode_shape *s, const float *q, const void *kbase, const void *vbase,
                         const void *const *kptrs, const void *const *vptrs, const float *ksbase,
                         const float *vsbase, const float *const *ksptrs, const float *const *vsptrs,
                         const int *lens, float *out, void *workspace, size_t workspace_bytes,
                         attn_stream_t stream) {
    long long rs;
    int st = check_decode(s, &rs);
    if (st) return st;
    if (s->n_seq == 0) return ATTN_OK;
    if (!q || !out) return set_error(ATTN_ERR_INVALID, "decode: NULL q/out");
    if (!aligned(q, 4) || !aligned(out, 4) || !aligned(lens, 4))
        return set_error(ATTN_ERR_INVALID, "decode: misaligned q/out/lens");
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    const size_t need = decode_workspace_bytes(s->n_seq, s->heads, s->head_dim, s->max_len, s->kv_dtype);
    if (workspace) {
        if (workspace_bytes < need || !aligned(workspace, 256))
            return set_error(ATTN_ERR_WORKSPACE, "decode: workspace needs %zu bytes (256-byte aligned), got %zu",
                             need, workspace_bytes);
    } else {
        workspace = internal_workspace(need, cs);
        if (!workspace) return set_error(ATTN_ERR_NOMEM, "decode: cannot allocate %zu-byte workspace", need);
    }
    DecodeLaunch L;
    L.n_seq = s->n_seq; L.heads = s->heads; L.head_dim = s->head_dim; L.kv_dtype = s->kv_dtype;
    L.max_len = s->max_len; L.row_stride = rs; L.cap = s->cap;
    L.q = q; L.kbase = kbase; L.vbase = vbase; L.kptrs = kptrs; L.vptrs = vptrs;
    L.ksbase = ksbase; L.vsbase = vsbase; L.ksptrs = ksptrs; L.vsptrs = vsptrs;
    L.lens = lens; L.out = out; L.ws = workspace; L.err = device_error_ptr(); L.stream = cs;
    if (!L.err) return set_error(ATTN_ERR_CUDA, "decode: no device error word");
    return launch_decode(L);
}

int attn_decode_ex(const attn_decode_shape *s, const float *q, const void *kcache, const void *vcache,
                   const float *kscale, const float *vscale, const int *lens, float *out,
                   void *workspace, size_t workspace_bytes, attn_stream_t stream) {
    if (!kcache || !vcache) return set_error(ATTN_ERR_INVALID, "decode: NULL cache");
    if (!aligned(kcache, 16) || !aligned(vcache, 16)) return set_error(ATTN_ERR_INVALID, "decode: caches must be 16-byte aligned");
    if (s && s->kv_dtype == ATTN_I8 && (!kscale || !vscale))
        return set_error(ATTN_ERR_INVALID, "decode: INT8 cache needs kscale and vscale");
    return decode_common(s, q, kcache, vcache, nullptr, nullptr, kscale, vscale, nullptr, nullptr, lens,
                         out, workspace, workspace_bytes, stream);
}

int attn_decode_ptrs_ex(const attn_decode_shape *s, const float *q, const void *const *kptrs,
                        const void *const *vptrs, const float *const *kscales,
                        const float *const *vscales, const int *lens, float *out, void *workspace,
                        size_t workspace_bytes, attn_stream_t stream) {
    if (!kptrs || !vptrs) return set_error(ATTN_ERR_INVALID, "decode: NULL pointer arrays");
    if (s && s->kv_dtype == ATTN_I8 && (!kscales || !vscales))
        return set_error(ATTN_ERR_INVALID, "decode: INT8 cache needs scale pointer arrays");
    return decode_common(s, q, nullptr, nullptr, kptrs, vptrs, nullptr, nullptr, kscales, vscales, lens,
                         out, workspace, workspace_bytes, stream);
}

int attn_cached_attention(const float *q, const float *kcache, const float *vcache, float *out, int pos,
                          int heads, int head_dim, long long row_stride, attn_stream_t stream) {
    if (pos < 0) return set_error(ATTN_ERR_INVALID, "cached_attention: pos %d < 0", pos);
    attn_decode_shape s;
    s.n_seq = 1; s.heads = heads; s.head_dim = head_dim; s.kv_dtype = ATTN_F32;
    s.row_stride = row_stride; s.cap = (long long)pos + 1; s.max_len = pos + 1;
    // lens == NULL: every sequence attends max_len = pos+1 rows (rows 0..pos)
    return attn_decode_ex(&s, q, kcache, vcache, nullptr, nullptr, nullptr, out, nullptr, 0, stream);
}

int attn_kv_quantize_int8(const float *x, long long rows, int heads, int head_dim, long long row_stride,
                          int8_t *codes, float *scales, attn_stream_t stream) {
    if (rows < 0 || heads < 1 || !head_dim_ok(head_dim))
        return set_error(ATTN_ERR_INVALID, "quantize: bad shape rows=%lld H=%d d=%d", rows, heads, head_dim);
    const long long rs = row_stride ? row_stride : (long long)heads * head_dim;
    if (rs < (long long)heads * head_dim) return set_error(ATTN_ERR_INVALID, "quantize: row_stride too small");
    if (rows == 0) return ATTN_OK;
    if (!x || !codes || !scales) return set_error(ATTN_ERR_INVALID, "quantize: NULL pointer");
    return launch_quantize_int8(x, rows, heads, head_dim, rs, codes, scales,
                                reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// device KV cache
// ---------------------------------------------------------------------------
int attn_kv_cache_alloc(attn_kv_cache *c, int n_layers, int cap, int heads, int head_dim, int kv_dtype) {
    if (!c || n_layers < 1 || n_layers > ATTN_MAX_LAYERS || cap < 1 || heads < 1 || !head_dim_ok(head_dim) ||
        (kv_dtype != ATTN_F32 && kv_dtype != ATTN_I8))
        return set_error(ATTN_ERR_INVALID, "kv_cache_alloc: bad arguments");
    memset(c, 0, sizeof *c);
    c->n_layers = n_layers; c->cap = cap; c->heads = heads; c->head_dim = head_dim; c->kv_dtype = kv_dtype;
    const size_t elems = (size_t)cap * heads * head_dim;
    const size_t esz = kv_dtype == ATTN_F32 ? 4 : 1;
    for (int l = 0; l < n_layers; l++) {
        if (cudaMalloc(&c->k[l], elems * esz) != cudaSuccess || cudaMalloc(&c->v[l], elems * esz) != cudaSuccess ||
            cudaMemset(c->k[l], 0, elems * esz) != cudaSuccess || cudaMemset(c->v[l], 0, elems * esz) != cudaSuccess) {
            attn_kv_cache_free(c);
            return set_error(ATTN_ERR_NOMEM, "kv_cache_alloc: out of device memory");
        }
        if (kv_dtype == ATTN_I8) {
            const size_t sb = (size_t)cap * heads * sizeof(float);
            if (cudaMalloc(&c->kscale[l], sb) != cudaSuccess || cudaMalloc(&c->vscale[l], sb) != cudaSuccess) {
                attn_kv_cache_free(c);
                return set_error(ATTN_ERR_NOMEM, "kv_cache_alloc: out of device memory");
            }
        }
    }
    return ATTN_OK;
}

int attn_kv_cache_free(attn_kv_cache *c) {
    if (!c) return set_error(ATTN_ERR_INVALID, "kv_cache_free: NULL");
    for (int l = 0; l < ATTN_MAX_LAYERS; l++) {
        if (c->k[l]) cudaFree(c->k[l]);
        if (c->v[l]) cudaFree(c->v[l]);
        if (c->kscale[l]) cudaFree(c->kscale[l]);
        if (c->vscale[l]) cudaFree(c->vscale[l]);
        c->k[l] = c->v[l] = nullptr;
        c->kscale[l] = c->vscale[l] = nullptr;
    }
    c->n_layers = 0;
    return ATTN_OK;
}

int attn_kv_cache_append(attn_kv_cache *c, int layer, int pos, const float *krow, const float *vrow,
                         attn_stream_t stream) {
    if (!c || layer < 0 || layer >= c->n_layers || pos < 0 || pos >= c->cap || !krow || !vrow)
        return set_error(ATTN_ERR_INVALID, "kv_cache_append: bad arguments");
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    const int hd = c->heads * c->head_dim;
    if (c->kv_dtype == ATTN_F32)
        return launch_append_f32(krow, vrow, static_cast<float *>(c->k[layer]) + (size_t)pos * hd,
                                 static_cast<float *>(c->v[layer]) + (size_t)pos * hd, hd, cs);
    int st = launch_quantize_int8(krow, 1, c->heads, c->head_dim, hd,
                                  static_cast<int8_t *>(c->k[layer]) + (size_t)pos * hd,
                                  c->kscale[layer] + (size_t)pos * c->heads, cs);
    if (st) return st;
    return launch_quantize_int8(vrow, 1, c->heads, c->head_dim, hd,
                                static_cast<int8_t *>(c->v[layer]) + (size_t)pos * hd,
                                c->vscale[layer] + (size_t)pos * c->heads, cs);
}

// ---------------------------------------------------------------------------
// multi-GPU partitioning
// ---------------------------------------------------------------------------
int attn_shard_range(long long n_units, int world, int rank, long long *begin, long long *end) {
    if (n_units < 0 || world < 1 || rank < 0 || rank >= world || !begin || !end)
        return set_error(ATTN_ERR_INVALID, "shard_range: bad arguments");
    const long long base = n_units / world, extra = n_units % world;
    *begin = rank * base + std::min<long long>(rank, extra);
    *end = *begin + base + (rank < extra ? 1 : 0);
    return ATTN_OK;
}

int attn_shard_lpt(const int *lens, int n_seq, int heads, int world, int *out_rank, long long *out_load) {
    if (!lens || n_seq < 0 || heads < 1 || world < 1 || !out_rank)
        return set_error(ATTN_ERR_INVALID, "shard_lpt: bad arguments");
    // units sorted by cost descending (ties: lower unit index first), each
    // given to the currently least-loaded rank (ties: lowest rank).
    std::vector<int> order(n_seq);
    for (int i = 0; i < n_seq; i++) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return lens[a] > lens[b]; });
    typedef std::pair<long long, int> Load;   // (load, rank)
    std::priority_queue<Load, std::vector<Load>, std::greater<Load>> pq;
    for (int r = 0; r < world; r++) pq.push(Load(0, r));
    std::vector<long long> load(world, 0);
    for (int si = 0; si < n_seq; si++) {
        const int sq = order[si];
        for (int h = 0; h < heads; h++) {
            Load top = pq.top();
            pq.pop();
            out_rank[(long long)sq * heads + h] = top.second;
            top.first += lens[sq];
            load[top.second] = top.first;
            pq.push(top);
        }
    }
    if (out_load)
        for (int r = 0; r < world; r++) out_load[r] = load[r];
    return ATTN_OK;
}

int attn_gather_permute(const void *staging, void *out, int world, int batch, int seq_len, int heads,
                        int head_dim, int dtype, attn_stream_t stream) {
    if (!staging || !out || world < 1 || batch < 0 || seq_len < 0 || heads < 1 || heads % world ||
        !head_dim_ok(head_dim) || (dtype != ATTN_F32 && dtype != ATTN_BF16))
        return set_error(ATTN_ERR_INVALID, "gather_permute: bad arguments");
    if (batch == 0 || seq_len == 0) return ATTN_OK;
    return launch_gather_permute(staging, out, world, batch, seq_len, heads, head_dim, dtype,
                                 reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
