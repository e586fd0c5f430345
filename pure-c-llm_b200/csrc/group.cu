// group.cu -- multi-GPU work split of the attention calls by (batch x head)
// units, and the NCCL gathers for callers that need an output whole.
//
// The reference has no multi-GPU code (its trainer, train_kaggle.cu:346, is one
// host process driving one GPU).  Attention has no exchange step between
// (batch, head) units, so the compute needs no collective: each GPU runs the
// ordinary kernels on its share.  NCCL (over NVLink) is the data plane of the
// gathers only, and no kernel here reads another GPU's memory.
//
// Two ways to drive a group:
//   * one host thread, several devices (the reference's single-process model):
//     attn_init(ngpus) creates one communicator per device with
//     ncclCommInitAll, and attn_fwd_multi / attn_decode_multi run every
//     device's share and gather in one call (collectives inside
//     ncclGroupStart/End);
//   * one process per GPU: attn_init_rank joins a communicator from a
//     128-byte id made by attn_get_unique_id on rank 0; each rank calls the
//     ordinary entry points on its share (attn_split_plan / attn_shard_lpt say
//     which) and attn_gather_split / attn_gather_rows to assemble outputs.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or $ATTN_NCCL_LIB), so
// single-GPU users of the library do not need it.  NVLS (in-switch reduction)
// is switched off unless the caller's environment says otherwise: a gather
// gains nothing from it.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "common.cuh"

namespace attn {

// staging [n][rows_local][cols_local] (16-byte chunks) -> out rows of the
// (B*T, H*d) layout: rank r = rb * nh + rh holds batches [rb*Bl, (rb+1)*Bl)
// and heads [rh*Hl, (rh+1)*Hl).
__global__ void grid_permute_kernel(const uint4 *__restrict__ staging, char *__restrict__ out, int n, int nh,
                                    long long rows_local, int T, int chunks_local, long long out_stride_bytes,
                                    int col_bytes_local)
{
    const long long total = (long long)n * rows_local * chunks_local;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(i % chunks_local);
        const long long t = i / chunks_local;
        const long long row = t % rows_local;
        const int r = (int)(t / rows_local);
        const int rb = r / nh, rh = r % nh;
        const long long grow = (long long)rb * rows_local + row;   // rows_local = Bl * T
        (void)T;
        uint4 *dst = reinterpret_cast<uint4 *>(out + grow * out_stride_bytes + (long long)rh * col_bytes_local) + c;
        *dst = staging[i];
    }
}

// staging rows (all ranks' padded blocks) -> out rows named by order[]
// (order[i] < 0: padding).
__global__ void scatter_rows_kernel(const uint4 *__restrict__ staging, uint4 *__restrict__ out,
                                    const int *__restrict__ order, long long n_rows, int chunks, int n_out)
{
    const long long total = n_rows * chunks;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / chunks;
        const int c = (int)(i % chunks);
        const int dst = __ldg(order + r);
        if (dst >= 0 && dst < n_out) out[(long long)dst * chunks + c] = staging[i];
    }
}

}  // namespace attn

namespace attn_host {

int set_error(int status, const char *fmt, ...);

// ---------------------------------------------------------------------------
// NCCL, resolved at run time
// ---------------------------------------------------------------------------
struct NcclApi {
    void *h = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommInitAll)(ncclComm_t *, int, const int *) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

static NcclApi g_nccl;
static std::mutex g_group_mu;

template <typename F>
static bool sym(void *h, const char *name, F &f) {
    f = reinterpret_cast<F>(dlsym(h, name));
    return f != nullptr;
}

static int load_nccl() {
    if (g_nccl.h) return ATTN_OK;
    const char *path = getenv("ATTN_NCCL_LIB");
    void *h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) return set_error(ATTN_ERR_UNSUPPORTED, "multi-GPU: cannot load NCCL (%s)", dlerror());
    NcclApi a;
    a.h = h;
    if (!sym(h, "ncclGetUniqueId", a.GetUniqueId) || !sym(h, "ncclCommInitRank", a.CommInitRank) ||
        !sym(h, "ncclCommInitAll", a.CommInitAll) || !sym(h, "ncclCommDestroy", a.CommDestroy) ||
        !sym(h, "ncclCommAbort", a.CommAbort) || !sym(h, "ncclCommGetAsyncError", a.CommGetAsyncError) ||
        !sym(h, "ncclAllGather", a.AllGather) || !sym(h, "ncclGroupStart", a.GroupStart) ||
        !sym(h, "ncclGroupEnd", a.GroupEnd) || !sym(h, "ncclGetErrorString", a.GetErrorString)) {
        dlclose(h);
        return set_error(ATTN_ERR_UNSUPPORTED, "multi-GPU: NCCL library lacks a required symbol");
    }
    g_nccl = a;
    return ATTN_OK;
}

static int nccl_fail(const char *what, ncclResult_t r) {
    return set_error(ATTN_ERR_COMM, "%s: %s", what, g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "NCCL error");
}

// ---------------------------------------------------------------------------
// the group
// ---------------------------------------------------------------------------
struct Group {
    int mode = 0;                    // 0 none, 1 one process drives all devices, 2 one process per rank
    int nranks = 0, rank = 0;        // rank: this process's rank (mode 2)
    std::vector<ncclComm_t> comms;   // mode 1: one per device; mode 2: one
    std::vector<int> devices;        // device of each comm
};
static Group g_group;

static void nvls_off_by_default() { setenv("NCCL_NVLS_ENABLE", "0", 0); }

static void teardown(bool abort_comms) {
    for (ncclComm_t c : g_group.comms) {
        if (!c) continue;
        if (abort_comms) g_nccl.CommAbort(c);
        else g_nccl.CommDestroy(c);
    }
    g_group = Group();
}

// ---------------------------------------------------------------------------
// split plan: nb x nh grid of ranks over (batch, head)
// ---------------------------------------------------------------------------
static int gcd_i(int a, int b) { while (b) { int t = a % b; a = b; b = t; } return a; }

static int plan(int batch, int heads, int nranks, int rank, attn_split *sp) {
    if (batch < 1 || heads < 1 || nranks < 1 || rank < 0 || rank >= nranks || !sp)
        return set_error(ATTN_ERR_INVALID, "split_plan: bad arguments (batch %d heads %d nranks %d rank %d)",
                         batch, heads, nranks, rank);
    // as many ranks along the batch as divide both (whole batches keep each
    // rank's rows contiguous), the rest along the heads
    int nb = 0;
    for (int c = gcd_i(batch, nranks); c >= 1 && !nb; c--)
        if (nranks % c == 0 && batch % c == 0 && heads % (nranks / c) == 0) nb = c;
    const int nh = nb ? nranks / nb : 0;
    if (!nb)
        return set_error(ATTN_ERR_UNSUPPORTED, "split_plan: %d ranks do not split %d batches x %d heads evenly",
                         nranks, batch, heads);
    sp->nb = nb;
    sp->nh = nh;
    sp->batch = batch / nb;
    sp->heads = heads / nh;
    sp->batch0 = (rank / nh) * sp->batch;
    sp->head0 = (rank % nh) * sp->heads;
    return ATTN_OK;
}

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

static int esize(int dtype) { return dtype == ATTN_BF16 ? 2 : 4; }

static int launch_grid_permute(const void *staging, void *out, int n, int nh, long long rows_local, int T,
                               long long col_bytes_local, long long out_stride_bytes, cudaStream_t s) {
    const int chunks = (int)(col_bytes_local / 16);
    const long long total = (long long)n * rows_local * chunks;
    if (total == 0) return ATTN_OK;
    const unsigned blocks = (unsigned)std::min<long long>((total + 255) / 256, 148LL * 16);
    attn::grid_permute_kernel<<<blocks, 256, 0, s>>>(static_cast<const uint4 *>(staging), static_cast<char *>(out),
                                                     n, nh, rows_local, T, chunks, out_stride_bytes,
                                                     (int)col_bytes_local);
    return check_launch("grid_permute_kernel");
}

}  // namespace attn_host

using namespace attn_host;

extern "C" {

int attn_get_unique_id(unsigned char id[128]) {
    if (!id) return set_error(ATTN_ERR_INVALID, "get_unique_id: NULL");
    std::lock_guard<std::mutex> lk(g_group_mu);
    int st = load_nccl();
    if (st) return st;
    ncclUniqueId u;
    ncclResult_t r = g_nccl.GetUniqueId(&u);
    if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
    static_assert(sizeof(u) == 128, "ncclUniqueId size");
    memcpy(id, &u, 128);
    return ATTN_OK;
}

int attn_init(int ngpus) {
    std::lock_guard<std::mutex> lk(g_group_mu);
    if (ngpus < 1) return set_error(ATTN_ERR_INVALID, "attn_init: ngpus %d", ngpus);
    if (g_group.mode) return set_error(ATTN_ERR_INVALID, "attn_init: a group exists (attn_finalize first)");
    int st = load_nccl();
    if (st) return st;
    nvls_off_by_default();
    std::vector<ncclComm_t> comms(ngpus, nullptr);
    std::vector<int> devs(ngpus);
    for (int i = 0; i < ngpus; i++) devs[i] = i;
    ncclResult_t r = g_nccl.CommInitAll(comms.data(), ngpus, devs.data());
    if (r != ncclSuccess) return nccl_fail("ncclCommInitAll", r);
    g_group.mode = 1;
    g_group.nranks = ngpus;
    g_group.comms = comms;
    g_group.devices = devs;
    return ATTN_OK;
}

int attn_init_rank(int nranks, int rank, int device, const unsigned char id[128]) {
    std::lock_guard<std::mutex> lk(g_group_mu);
    if (nranks < 1 || rank < 0 || rank >= nranks || !id)
        return set_error(ATTN_ERR_INVALID, "attn_init_rank: nranks %d rank %d", nranks, rank);
    if (g_group.mode) return set_error(ATTN_ERR_INVALID, "attn_init_rank: a group exists (attn_finalize first)");
    int st = load_nccl();
    if (st) return st;
    nvls_off_by_default();
    if (device >= 0) {
        cudaError_t e = cudaSetDevice(device);
        if (e != cudaSuccess) return set_error(ATTN_ERR_CUDA, "attn_init_rank: cudaSetDevice(%d): %s", device,
                                               cudaGetErrorString(e));
    }
    int dev = device;
    if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    ncclUniqueId u;
    memcpy(&u, id, 128);
    ncclComm_t c = nullptr;
    ncclResult_t r = g_nccl.CommInitRank(&c, nranks, u, rank);
    if (r != ncclSuccess) return nccl_fail("ncclCommInitRank", r);
    g_group.mode = 2;
    g_group.nranks = nranks;
    g_group.rank = rank;
    g_group.comms = {c};
    g_group.devices = {dev};
    return ATTN_OK;
}

int attn_finalize(void) {
    std::lock_guard<std::mutex> lk(g_group_mu);
    if (!g_group.mode) return ATTN_OK;
    teardown(false);
    return ATTN_OK;
}

int attn_group_size(void) {
    std::lock_guard<std::mutex> lk(g_group_mu);
    return g_group.mode ? g_group.nranks : 0;
}

int attn_group_sync(const attn_stream_t *streams, int n_streams, int timeout_ms) {
    if (n_streams < 0 || (n_streams > 0 && !streams) || timeout_ms < 0)
        return set_error(ATTN_ERR_INVALID, "group_sync: bad arguments");
    std::lock_guard<std::mutex> lk(g_group_mu);
    if (!g_group.mode) return set_error(ATTN_ERR_INVALID, "group_sync: no group");
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<char> done(n_streams, 0);
    while (true) {
        for (size_t i = 0; i < g_group.comms.size(); i++) {
            ncclResult_t ar = ncclSuccess;
            ncclResult_t r = g_nccl.CommGetAsyncError(g_group.comms[i], &ar);
            if (r != ncclSuccess || (ar != ncclSuccess && ar != ncclInProgress)) {
                const ncclResult_t bad = r != ncclSuccess ? r : ar;
                const int st = set_error(ATTN_ERR_COMM, "group_sync: communicator %zu failed (%s); the group was "
                                         "aborted", i, g_nccl.GetErrorString(bad));
                teardown(true);
                return st;
            }
        }
        bool all = true;
        for (int i = 0; i < n_streams; i++) {
            if (done[i]) continue;
            cudaError_t e = cudaStreamQuery(reinterpret_cast<cudaStream_t>(streams[i]));
            if (e == cudaSuccess) done[i] = 1;
            else if (e == cudaErrorNotReady) all = false;
            else return set_error(ATTN_ERR_CUDA, "group_sync: stream %d: %s", i, cudaGetErrorString(e));
        }
        if (all) return ATTN_OK;
        const long long ms = std::chrono::duration_cast<std::chrono::milliseconds>(
            std::chrono::steady_clock::now() - t0).count();
        if (ms > timeout_ms) {
            const int st = set_error(ATTN_ERR_COMM, "group_sync: streams not done after %d ms; the group was aborted",
                                     timeout_ms);
            teardown(true);
            return st;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

int attn_split_plan(int batch, int heads, int nranks, int rank, attn_split *out) {
    return plan(batch, heads, nranks, rank, out);
}

size_t attn_gather_workspace_bytes(const attn_shape *s, int dtype, int nranks) {
    if (!s || nranks < 1) return 0;
    attn_split sp;
    if (plan(s->batch, s->heads, nranks, 0, &sp)) return 0;
    if (sp.nh == 1) return 0;
    const size_t local = (size_t)sp.batch * s->seq_len * sp.heads * s->head_dim * esize(dtype);
    return align256(local) + align256(local * nranks);
}

int attn_gather_split(const attn_shape *s, int dtype, const void *local, void *out, void *ws, size_t ws_bytes,
                      attn_stream_t stream) {
    std::lock_guard<std::mutex> lk(g_group_mu);
    if (g_group.mode != 2)
        return set_error(ATTN_ERR_INVALID, "gather_split: needs a one-process-per-rank group (attn_init_rank); a "
                         "single-process group gathers inside attn_fwd_multi");
    if (!s || !local || !out || (dtype != ATTN_F32 && dtype != ATTN_BF16))
        return set_error(ATTN_ERR_INVALID, "gather_split: bad arguments");
    attn_split sp;
    int st = plan(s->batch, s->heads, g_group.nranks, g_group.rank, &sp);
    if (st) return st;
    const int es = esize(dtype);
    const long long hd = (long long)s->heads * s->head_dim;
    const long long ors = s->out_row_stride ? s->out_row_stride : hd;
    const size_t local_bytes = (size_t)sp.batch * s->seq_len * sp.heads * s->head_dim * es;
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    ncclComm_t comm = g_group.comms[0];
    if (sp.nh == 1) {
        if (ors != hd) return set_error(ATTN_ERR_INVALID, "gather_split: whole-batch gather needs dense output rows");
        ncclResult_t r = g_nccl.AllGather(local, out, local_bytes, ncclUint8, comm, cs);
        return r == ncclSuccess ? ATTN_OK : nccl_fail("ncclAllGather", r);
    }
    if (((uintptr_t)out | (uintptr_t)ws) & 15 || (ors * es) % 16)
        return set_error(ATTN_ERR_INVALID, "gather_split: output and workspace must be 16-byte aligned");
    const size_t need = align256(local_bytes) + align256(local_bytes * g_group.nranks);
    if (!ws || ws_bytes < need)
        return set_error(ATTN_ERR_WORKSPACE, "gather_split: workspace needs %zu bytes, got %zu", need, ws_bytes);
    char *stg = static_cast<char *>(ws) + align256(local_bytes);
    ncclResult_t r = g_nccl.AllGather(local, stg, local_bytes, ncclUint8, comm, cs);
    if (r != ncclSuccess) return nccl_fail("ncclAllGather", r);
    return launch_grid_permute(stg, out, g_group.nranks, sp.nh, (long long)sp.batch * s->seq_len, s->seq_len,
                               (long long)sp.heads * s->head_dim * es, ors * es, cs);
}

size_t attn_gather_rows_workspace_bytes(int max_local, size_t row_bytes, int nranks) {
    if (max_local < 0 || nranks < 1) return 0;
    return align256((size_t)max_local * row_bytes * nranks);
}

int attn_gather_rows(const void *local, int max_local, size_t row_bytes, const int *order, int n_out, void *out,
                     void *ws, size_t ws_bytes, attn_stream_t stream) {
    std::lock_guard<std::mutex> lk(g_group_mu);
    if (g_group.mode != 2)
        return set_error(ATTN_ERR_INVALID, "gather_rows: needs a one-process-per-rank group (attn_init_rank); a "
                         "single-process group gathers inside attn_decode_multi");
    if (!local || !out || max_local < 0 || n_out < 0 || row_bytes == 0 || row_bytes % 16 ||
        (((uintptr_t)local | (uintptr_t)out) & 15))
        return set_error(ATTN_ERR_INVALID, "gather_rows: bad arguments (rows of a multiple of 16 bytes, 16-byte "
                         "aligned buffers)");
    cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);
    ncclComm_t comm = g_group.comms[0];
    const size_t bytes = (size_t)max_local * row_bytes;
    if (!order) {
        if ((long long)n_out != (long long)max_local * g_group.nranks)
            return set_error(ATTN_ERR_INVALID, "gather_rows: without an order, n_out must be nranks * max_local");
        ncclResult_t r = g_nccl.AllGather(local, out, bytes, ncclUint8, comm, cs);
        return r == ncclSuccess ? ATTN_OK : nccl_fail("ncclAllGather", r);
    }
    const size_t need = attn_gather_rows_workspace_bytes(max_local, row_bytes, g_group.nranks);
    if (!ws || ws_bytes < need || ((uintptr_t)ws & 15))
        return set_error(ATTN_ERR_WORKSPACE, "gather_rows: workspace needs %zu bytes, got %zu", need, ws_bytes);
    ncclResult_t r = g_nccl.AllGather(local, ws, bytes, ncclUint8, comm, cs);
    if (r != ncclSuccess) return nccl_fail("ncclAllGather", r);
    const long long n_rows = (long long)max_local * g_group.nranks;
    const int chunks = (int)(row_bytes / 16);
    const long long total = n_rows * chunks;
    if (total == 0) return ATTN_OK;
    const unsigned blocks = (unsigned)std::min<long long>((total + 255) / 256, 148LL * 16);
    attn::scatter_rows_kernel<<<blocks, 256, 0, cs>>>(static_cast<const uint4 *>(ws), static_cast<uint4 *>(out), order,
                                                       n_rows, chunks, n_out);
    return check_launch("scatter_rows_kernel");
}

// ---------------------------------------------------------------------------
// one host thread, all devices of an attn_init group
// ---------------------------------------------------------------------------
int attn_fwd_multi(const attn_shape *s, int dtype, const void *const *q, const void *const *k,
                   const void *const *v, void *const *o, float *const *lse, int gather, void *const *ws,
                   const size_t *ws_bytes, const attn_stream_t *streams) {
    std::lock_guard<std::mutex> lk(g_group_mu);
    if (g_group.mode != 1) return set_error(ATTN_ERR_INVALID, "fwd_multi: needs an attn_init group");
    if (!s || !q || !k || !v || !o || !streams || (dtype != ATTN_F32 && dtype != ATTN_BF16))
        return set_error(ATTN_ERR_INVALID, "fwd_multi: bad arguments");
    const int n = g_group.nranks, es = esize(dtype);
    const long long hd = (long long)s->heads * s->head_dim;
    const long long irs = s->in_row_stride ? s->in_row_stride : hd;
    const long long ors = s->out_row_stride ? s->out_row_stride : hd;
    int caller_dev = 0;
    cudaGetDevice(&caller_dev);
    std::vector<attn_split> sp(n);
    for (int g = 0; g < n; g++) {
        int st = plan(s->batch, s->heads, n, g, &sp[g]);
        if (st) return st;
    }
    const bool packed = gather && sp[0].nh > 1;
    const size_t local_bytes = (size_t)sp[0].batch * s->seq_len * sp[0].heads * s->head_dim * es;
    if (gather && !packed && ors != hd)
        return set_error(ATTN_ERR_INVALID, "fwd_multi: a whole-batch gather needs dense output rows");
    if (packed) {
        const size_t need = align256(local_bytes) + align256(local_bytes * n);
        for (int g = 0; g < n; g++)
            if (!ws || !ws[g] || !ws_bytes || ws_bytes[g] < need)
                return set_error(ATTN_ERR_WORKSPACE, "fwd_multi: device %d workspace needs %zu bytes", g, need);
    }
    int st = ATTN_OK;
    for (int g = 0; g < n && !st; g++) {
        cudaSetDevice(g_group.devices[g]);
        const attn_split &p = sp[g];
        attn_shape ls = *s;
        ls.batch = p.batch;
        ls.heads = p.heads;
        ls.in_row_stride = irs;
        const long long in_off = ((long long)p.batch0 * s->seq_len * irs + (long long)p.head0 * s->head_dim) * es;
        void *dst;
        if (packed) {
            ls.out_row_stride = (long long)p.heads * s->head_dim;
            dst = ws[g];
        } else {
            ls.out_row_stride = ors;
            dst = static_cast<char *>(o[g]) + ((long long)p.batch0 * s->seq_len * ors + (long long)p.head0 * s->head_dim) * es;
        }
        st = attn_fwd_ex(&ls, dtype, static_cast<const char *>(q[g]) + in_off, static_cast<const char *>(k[g]) + in_off,
                         static_cast<const char *>(v[g]) + in_off, dst, lse ? lse[g] : nullptr, streams[g]);
    }
    if (!st && gather) {
        ncclResult_t r = g_nccl.GroupStart();
        for (int g = 0; g < n && r == ncclSuccess; g++) {
            const attn_split &p = sp[g];
            cudaStream_t cs = reinterpret_cast<cudaStream_t>(streams[g]);
            if (packed) {
                r = g_nccl.AllGather(ws[g], static_cast<char *>(ws[g]) + align256(local_bytes), local_bytes, ncclUint8,
                                     g_group.comms[g], cs);
            } else {
                char *base = static_cast<char *>(o[g]);
                r = g_nccl.AllGather(base + (long long)p.batch0 * s->seq_len * hd * es, base, local_bytes, ncclUint8,
                                     g_group.comms[g], cs);
            }
        }
        ncclResult_t r2 = g_nccl.GroupEnd();
        if (r != ncclSuccess || r2 != ncclSuccess) st = nccl_fail("fwd_multi: all-gather", r != ncclSuccess ? r : r2);
        for (int g = 0; g < n && !st && packed; g++) {
            cudaSetDevice(g_group.devices[g]);
            st = launch_grid_permute(static_cast<char *>(ws[g]) + align256(local_bytes), o[g], n, sp[g].nh,
                                     (long long)sp[g].batch * s->seq_len, s->seq_len,
                                     (long long)sp[g].heads * s->head_dim * es, ors * es,
                                     reinterpret_cast<cudaStream_t>(streams[g]));
        }
    }
    cudaSetDevice(caller_dev);
    return st;
}

int attn_decode_multi(const attn_decode_shape *shapes, const float *const *q, const void *const *kcache,
                      const void *const *vcache, const float *const *kscale, const float *const *vscale,
                      const int *const *lens, float *const *out, int gather, int max_local,
                      const int *const *order, int n_total, float *const *out_full, void *const *ws,
                      const size_t *ws_bytes, const attn_stream_t *streams) {
    std::lock_guard<std::mutex> lk(g_group_mu);
    if (g_group.mode != 1) return set_error(ATTN_ERR_INVALID, "decode_multi: needs an attn_init group");
    if (!shapes || !q || !kcache || !vcache || !out || !streams)
        return set_error(ATTN_ERR_INVALID, "decode_multi: bad arguments");
    const int n = g_group.nranks;
    for (int g = 0; g < n; g++)
        if (shapes[g].n_seq > max_local || shapes[g].heads != shapes[0].heads ||
            shapes[g].head_dim != shapes[0].head_dim)
            return set_error(ATTN_ERR_INVALID, "decode_multi: device %d has %d sequences (max_local %d) or another "
                             "head shape", g, shapes[g].n_seq, max_local);
    const size_t row_bytes = (size_t)shapes[0].heads * shapes[0].head_dim * sizeof(float);
    const size_t need = align256((size_t)max_local * row_bytes * n);
    if (gather) {
        if (!order || !out_full || !ws || !ws_bytes)
            return set_error(ATTN_ERR_INVALID, "decode_multi: a gather needs order, out_full and ws");
        for (int g = 0; g < n; g++)
            if (!ws[g] || ws_bytes[g] < need || !order[g] || !out_full[g])
                return set_error(ATTN_ERR_WORKSPACE, "decode_multi: device %d gather workspace needs %zu bytes", g,
                                 need);
    }
    int caller_dev = 0;
    cudaGetDevice(&caller_dev);
    int st = ATTN_OK;
    for (int g = 0; g < n && !st; g++) {
        cudaSetDevice(g_group.devices[g]);
        if (shapes[g].n_seq == 0) continue;
        st = attn_decode_ex(&shapes[g], q[g], kcache[g], vcache[g], kscale ? kscale[g] : nullptr,
                            vscale ? vscale[g] : nullptr, lens ? lens[g] : nullptr, out[g], nullptr, 0, streams[g]);
    }
    if (!st && gather) {
        ncclResult_t r = g_nccl.GroupStart();
        for (int g = 0; g < n && r == ncclSuccess; g++)
            r = g_nccl.AllGather(out[g], ws[g], (size_t)max_local * row_bytes, ncclUint8, g_group.comms[g],
                                 reinterpret_cast<cudaStream_t>(streams[g]));
        ncclResult_t r2 = g_nccl.GroupEnd();
        if (r != ncclSuccess || r2 != ncclSuccess) st = nccl_fail("decode_multi: all-gather", r != ncclSuccess ? r : r2);
        const long long n_rows = (long long)max_local * n;
        const int chunks = (int)(row_bytes / 16);
        for (int g = 0; g < n && !st && n_rows > 0; g++) {
            cudaSetDevice(g_group.devices[g]);
            const unsigned blocks = (unsigned)std::min<long long>((n_rows * chunks + 255) / 256, 148LL * 16);
            attn::scatter_rows_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(streams[g])>>>(
                static_cast<const uint4 *>(ws[g]), reinterpret_cast<uint4 *>(out_full[g]), order[g], n_rows, chunks,
                n_total);
            st = check_launch("scatter_rows_kernel");
        }
    }
    cudaSetDevice(caller_dev);
    return st;
}

}  // extern "C"
