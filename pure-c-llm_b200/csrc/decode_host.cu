// decode_host.cu -- KV-cached decode attention for callers whose caches live
// in host memory: the CPU generators (transformer.c's forward_block, whose
// static cached_attention is transformer.c:203-248, and generate.c's inline
// copy at generate.c:130-152).
//
// The caller keeps its host cache and its own argument list; the library
// keeps a device mirror of each host cache (keyed by the pair of host K/V
// pointers) and, on every call, copies over only the rows it has not seen
// (the generator writes row `pos` just before attending, transformer.c:256-264),
// then runs the GPU decode on the mirror and copies the output row back.  A
// call whose pos is below the mirrored length (a new sequence in the same
// buffers) re-copies rows from pos onward; rows below a call's pos are taken
// to be unchanged since they were mirrored, as the reference's generators
// never rewrite them.
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace attn_host {

struct Mirror {
    int device = -1;
    float *k = nullptr, *v = nullptr;       // cap x row_stride
    float *q = nullptr, *o = nullptr;       // one row each
    long long row_stride = 0;
    int cap = 0, heads = 0, head_dim = 0;
    int rows = 0;                           // rows [0, rows) mirrored
};

static std::mutex g_host_mu;
static std::map<std::pair<const float *, const float *>, Mirror> g_mirrors;
// transformer.h:35-38 (T_MAX 512, N_HEADS 16, D_HEAD 96; D_MODEL = 16 * 96)
static int g_dec_heads = 16, g_dec_head_dim = 96, g_dec_tmax = 512;

static void free_mirror(Mirror &m) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(m.device);
    cudaFree(m.k);
    cudaFree(m.v);
    cudaFree(m.q);
    cudaFree(m.o);
    cudaSetDevice(prev);
    m = Mirror();
}

static int host_decode(const float *q, const float *kc, const float *vc, float *out, int pos, int heads,
                       int head_dim, long long row_stride, int cap) {
    if (!q || !kc || !vc || !out || heads < 1 || cap < 1 || pos < 0 || pos >= cap)
        return set_error(ATTN_ERR_INVALID, "cached_attention_host: bad arguments (pos %d, cap %d)", pos, cap);
    const long long hd = (long long)heads * head_dim;
    if (row_stride == 0) row_stride = hd;
    if (row_stride < hd || row_stride % 4)
        return set_error(ATTN_ERR_INVALID, "cached_attention_host: row_stride %lld", row_stride);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return set_error(ATTN_ERR_CUDA, "cached_attention_host: no device");
    std::lock_guard<std::mutex> lk(g_host_mu);
    Mirror &m = g_mirrors[std::make_pair(kc, vc)];
    if (m.k && (m.device != dev || m.cap != cap || m.row_stride != row_stride || m.heads != heads ||
                m.head_dim != head_dim))
        free_mirror(m);
    if (!m.k) {
        const size_t bytes = (size_t)cap * row_stride * sizeof(float);
        if (cudaMalloc(&m.k, bytes) != cudaSuccess || cudaMalloc(&m.v, bytes) != cudaSuccess ||
            cudaMalloc(&m.q, hd * sizeof(float)) != cudaSuccess || cudaMalloc(&m.o, hd * sizeof(float)) != cudaSuccess) {
            m.device = dev;
            free_mirror(m);
            return set_error(ATTN_ERR_NOMEM, "cached_attention_host: cannot allocate a %zu-byte cache mirror", bytes);
        }
        m.device = dev;
        m.cap = cap;
        m.row_stride = row_stride;
        m.heads = heads;
        m.head_dim = head_dim;
        m.rows = 0;
    }
    // rows the mirror lacks: [min(rows, pos), pos]; row pos is always re-sent
    const int r0 = m.rows < pos ? m.rows : pos;
    const size_t off = (size_t)r0 * row_stride, n = (size_t)(pos + 1 - r0) * row_stride;
    cudaStream_t s = nullptr;   // legacy default stream, as the reference's GPU code
    cudaError_t e = cudaMemcpyAsync(m.k + off, kc + off, n * sizeof(float), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m.v + off, vc + off, n * sizeof(float), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m.q, q, hd * sizeof(float), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return set_error(ATTN_ERR_CUDA, "cached_attention_host: copy in: %s", cudaGetErrorString(e));
    m.rows = pos + 1;
    attn_decode_shape ds;
    ds.n_seq = 1;
    ds.heads = heads;
    ds.head_dim = head_dim;
    ds.kv_dtype = ATTN_F32;
    ds.row_stride = row_stride;
    ds.cap = cap;
    ds.max_len = pos + 1;
    int st = attn_decode_ex(&ds, m.q, m.k, m.v, nullptr, nullptr, nullptr, m.o, nullptr, 0, nullptr);
    if (st) return st;
    e = cudaMemcpy(out, m.o, hd * sizeof(float), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return set_error(ATTN_ERR_CUDA, "cached_attention_host: copy out: %s", cudaGetErrorString(e));
    return ATTN_OK;
}

}  // namespace attn_host

using namespace attn_host;

extern "C" {

int attn_set_decode_macro_shape(int heads, int head_dim, int t_max) {
    if (heads < 1 || t_max < 1 || !(head_dim == 32 || head_dim == 64 || head_dim == 96 || head_dim == 128))
        return set_error(ATTN_ERR_INVALID, "bad decode macro shape H=%d d=%d T_MAX=%d", heads, head_dim, t_max);
    std::lock_guard<std::mutex> lk(g_host_mu);
    g_dec_heads = heads;
    g_dec_head_dim = head_dim;
    g_dec_tmax = t_max;
    return ATTN_OK;
}

void attn_cached_attention_host(const float *q, const float *kcache, const float *vcache, float *out,
                                float *scores, int pos) {
    (void)scores;   // the reference's score scratch; the GPU keeps its scores on chip
    int heads, head_dim, tmax;
    {
        std::lock_guard<std::mutex> lk(g_host_mu);
        heads = g_dec_heads;
        head_dim = g_dec_head_dim;
        tmax = g_dec_tmax;
    }
    const int st = host_decode(q, kcache, vcache, out, pos, heads, head_dim, 0, tmax);
    if (st) {
        fprintf(stderr, "CUDA error '%s' at attn_cached_attention_host\n", attn_last_error());
        exit(1);
    }
}

int attn_cached_attention_host_ex(const float *q, const float *kcache, const float *vcache, float *out, int pos,
                                  int heads, int head_dim, long long row_stride, int cap) {
    return host_decode(q, kcache, vcache, out, pos, heads, head_dim, row_stride, cap);
}

int attn_host_cache_release(const float *kcache, const float *vcache) {
    std::lock_guard<std::mutex> lk(g_host_mu);
    auto it = g_mirrors.find(std::make_pair(kcache, vcache));
    if (it == g_mirrors.end()) return ATTN_OK;
    free_mirror(it->second);
    g_mirrors.erase(it);
    return ATTN_OK;
}

}  // extern "C"
