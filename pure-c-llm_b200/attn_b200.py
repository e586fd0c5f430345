"""ctypes binding of libattn_b200.so -- the host-side mirror of the C ABI
declared in include/attn_b200.h.

The names follow the reference's call surface (attn_fwd / attn_bwd of
gpu_kernels.h:67-72, cached_attention of transformer.c:203).  Raw-pointer
wrappers take integer device addresses; the `*_t` helpers take torch CUDA
tensors, which serve only as device memory and stream plumbing.  There is
no fallback: if the shared library is missing, importing this module raises.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libattn_b200.so")

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_NOMEM, ERR_WORKSPACE, ERR_DEVICE, ERR_COMM = range(8)
PROBS_LSE_OUT, PROBS_LSE = 0, 1      # attn_set_probs_mode
F32, BF16, I8 = 0, 1, 2
MAX_LAYERS = 64
STATIC_SCRATCH_BYTES = 4 << 20      # ATTN_DECODE_STATIC_SCRATCH_BYTES


class AttnError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"attn status {status}: {msg}")
        self.status = status


if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is not built; run `make -C pure-c-llm_b200` (or __graft_entry__.build())")
lib = ctypes.CDLL(LIB_PATH)


class Shape(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int), ("heads", ctypes.c_int), ("seq_len", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("in_row_stride", ctypes.c_longlong),
                ("out_row_stride", ctypes.c_longlong)]


class DecodeShape(ctypes.Structure):
    _fields_ = [("n_seq", ctypes.c_int), ("heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("kv_dtype", ctypes.c_int), ("row_stride", ctypes.c_longlong),
                ("cap", ctypes.c_longlong), ("max_len", ctypes.c_int)]


class KVCache(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("cap", ctypes.c_int), ("heads", ctypes.c_int),
                ("head_dim", ctypes.c_int), ("kv_dtype", ctypes.c_int),
                ("k", ctypes.c_void_p * MAX_LAYERS), ("v", ctypes.c_void_p * MAX_LAYERS),
                ("kscale", ctypes.c_void_p * MAX_LAYERS), ("vscale", ctypes.c_void_p * MAX_LAYERS)]


class QKVShape(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int), ("in_features", ctypes.c_int), ("out_features", ctypes.c_int),
                ("x_row_stride", ctypes.c_longlong), ("out_row_stride", ctypes.c_longlong)]


class Split(ctypes.Structure):
    _fields_ = [("batch0", ctypes.c_int), ("batch", ctypes.c_int), ("head0", ctypes.c_int),
                ("heads", ctypes.c_int), ("nb", ctypes.c_int), ("nh", ctypes.c_int)]


P = ctypes.c_void_p
I = ctypes.c_int
LL = ctypes.c_longlong
SZ = ctypes.c_size_t

# name -> (restype, argtypes); every symbol of include/attn_b200.h
SIGNATURES = {
    "attn_last_error": (ctypes.c_char_p, []),
    "attn_device_error": (I, [I, ctypes.POINTER(I)]),
    "attn_version": (I, []),
    "attn_fwd": (None, [P, P, P, P, P]),
    "attn_bwd": (None, [P, P, P, P, P, P, P, P, P]),
    "attn_set_macro_shape": (I, [I, I, I, I]),
    "attn_set_probs_mode": (I, [I]),
    "attn_fwd_ex": (I, [ctypes.POINTER(Shape), I, P, P, P, P, P, P]),
    "attn_bwd_workspace_bytes": (SZ, [ctypes.POINTER(Shape), I]),
    "attn_bwd_ex": (I, [ctypes.POINTER(Shape), I, P, P, P, P, P, P, P, P, P, I, P, SZ, P]),
    "attn_bwd_tc_workspace_bytes": (SZ, [ctypes.POINTER(Shape)]),
    "attn_qkv_workspace_bytes": (SZ, [ctypes.POINTER(QKVShape)]),
    "attn_qkv_proj_ex": (I, [ctypes.POINTER(QKVShape), P, P, P, P, P, P, P, P, P, P, P, SZ, P]),
    "attn_qkv_proj": (None, [P, P, P, P, P, P, P, P, P, P, I, I, I]),
    "attn_decode_workspace_bytes": (SZ, [ctypes.POINTER(DecodeShape)]),
    "attn_decode_ex": (I, [ctypes.POINTER(DecodeShape), P, P, P, P, P, P, P, P, SZ, P]),
    "attn_decode_ptrs_ex": (I, [ctypes.POINTER(DecodeShape), P, P, P, P, P, P, P, P, SZ, P]),
    "attn_decode_static_ex": (I, [ctypes.POINTER(DecodeShape), P, P, P, P, P, P, P, P]),
    "attn_cached_attention": (I, [P, P, P, P, I, I, I, LL, P]),
    "attn_kv_quantize_int8": (I, [P, LL, I, I, LL, P, P, P]),
    "attn_kv_cache_alloc": (I, [ctypes.POINTER(KVCache), I, I, I, I, I]),
    "attn_kv_cache_free": (I, [ctypes.POINTER(KVCache)]),
    "attn_kv_cache_append": (I, [ctypes.POINTER(KVCache), I, I, P, P, P]),
    "attn_shard_range": (I, [LL, I, I, ctypes.POINTER(LL), ctypes.POINTER(LL)]),
    "attn_shard_lpt": (I, [P, I, I, I, P, P]),
    "attn_gather_permute": (I, [P, P, I, I, I, I, I, I, P]),
    "attn_debug_decode_timeout": (I, [I, LL]),
    "attn_debug_qkv_timeout": (I, [I, LL]),
    "attn_cached_attention_host": (None, [P, P, P, P, P, I]),
    "attn_set_decode_macro_shape": (I, [I, I, I]),
    "attn_cached_attention_host_ex": (I, [P, P, P, P, I, I, I, LL, I]),
    "attn_host_cache_release": (I, [P, P]),
    "attn_init": (I, [I]),
    "attn_get_unique_id": (I, [P]),
    "attn_init_rank": (I, [I, I, I, P]),
    "attn_finalize": (I, []),
    "attn_group_size": (I, []),
    "attn_group_sync": (I, [P, I, I]),
    "attn_split_plan": (I, [I, I, I, I, ctypes.POINTER(Split)]),
    "attn_gather_workspace_bytes": (SZ, [ctypes.POINTER(Shape), I, I]),
    "attn_gather_split": (I, [ctypes.POINTER(Shape), I, P, P, P, SZ, P]),
    "attn_gather_rows_workspace_bytes": (SZ, [I, SZ, I]),
    "attn_gather_rows": (I, [P, I, SZ, P, I, P, P, SZ, P]),
    "attn_fwd_multi": (I, [ctypes.POINTER(Shape), I, P, P, P, P, P, I, P, P, P]),
    "attn_decode_multi": (I, [ctypes.POINTER(DecodeShape), P, P, P, P, P, P, P, I, I, P, I, P, P, P, P]),
}
for _name, (_res, _args) in SIGNATURES.items():
    _f = getattr(lib, _name)
    _f.restype = _res
    _f.argtypes = _args


def last_error() -> str:
    return lib.attn_last_error().decode()


def check(status: int):
    if status != OK:
        raise AttnError(status, last_error())


# ---------------------------------------------------------------------------
# raw-pointer API
# ---------------------------------------------------------------------------
def fwd_ex(shape: Shape, dtype, q, k, v, o, lse, stream=0):
    check(lib.attn_fwd_ex(ctypes.byref(shape), dtype, q, k, v, o, lse, stream))


def bwd_workspace_bytes(shape: Shape, dtype) -> int:
    return lib.attn_bwd_workspace_bytes(ctypes.byref(shape), dtype)


def bwd_ex(shape: Shape, dtype, do, q, k, v, o, lse, dq, dk, dv, accumulate, ws, ws_bytes, stream=0):
    check(lib.attn_bwd_ex(ctypes.byref(shape), dtype, do, q, k, v, o, lse, dq, dk, dv,
                          int(accumulate), ws, ws_bytes, stream))


def decode_workspace_bytes(shape: DecodeShape) -> int:
    return lib.attn_decode_workspace_bytes(ctypes.byref(shape))


def decode_ex(shape: DecodeShape, q, kc, vc, ks, vs, lens, out, ws=None, ws_bytes=0, stream=0):
    check(lib.attn_decode_ex(ctypes.byref(shape), q, kc, vc, ks, vs, lens, out, ws, ws_bytes, stream))


def shard_range(n_units: int, world: int, rank: int):
    b, e = LL(), LL()
    check(lib.attn_shard_range(n_units, world, rank, ctypes.byref(b), ctypes.byref(e)))
    return b.value, e.value


def split_plan(batch: int, heads: int, nranks: int, rank: int) -> Split:
    sp = Split()
    check(lib.attn_split_plan(batch, heads, nranks, rank, ctypes.byref(sp)))
    return sp


def shard_lpt(lens, heads: int, world: int):
    """LPT assignment of (seq, head) units; returns (rank per unit, load per rank)."""
    import numpy as np
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    ranks = np.empty(len(lens) * heads, dtype=np.int32)
    load = np.empty(world, dtype=np.int64)
    check(lib.attn_shard_lpt(lens.ctypes.data, len(lens), heads, world, ranks.ctypes.data, load.ctypes.data))
    return ranks, load


# ---------------------------------------------------------------------------
# torch-tensor helpers (device memory + stream plumbing only)
# ---------------------------------------------------------------------------
def _dtype_code(t):
    import torch
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise TypeError(f"unsupported dtype {t.dtype}")


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def forward_t(q, k, v, heads: int, batch: int, out=None, lse=None, want_lse=True):
    """q,k,v: (batch*T, heads*d) CUDA tensors (fp32 or bf16), row-major."""
    import torch
    rows, width = q.shape
    T = rows // batch
    d = width // heads
    out = torch.empty_like(q) if out is None else out
    if want_lse and lse is None:
        lse = torch.empty(batch * heads * T, dtype=torch.float32, device=q.device)
    shape = Shape(batch, heads, T, d, q.stride(0), out.stride(0))
    fwd_ex(shape, _dtype_code(q), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
           lse.data_ptr() if lse is not None else None, _stream())
    return out, lse


def backward_t(do, q, k, v, o, lse, heads: int, batch: int, dq=None, dk=None, dv=None, accumulate=False):
    import torch
    rows, width = q.shape
    T = rows // batch
    d = width // heads
    shape = Shape(batch, heads, T, d, q.stride(0), o.stride(0))
    dq = torch.zeros_like(q) if dq is None else dq
    dk = torch.zeros_like(q) if dk is None else dk
    dv = torch.zeros_like(q) if dv is None else dv
    nbytes = bwd_workspace_bytes(shape, _dtype_code(q))
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    bwd_ex(shape, _dtype_code(q), do.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
           lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), accumulate, ws.data_ptr(), nbytes,
           _stream())
    return dq, dk, dv


def qkv_proj_t(x, wq, wk, wv, bq=None, bk=None, bv=None, fused=False, out=None, workspace=None):
    """Q, K, V = x @ W + b for the three weights in one launch (train_kaggle.cu:152-154).
    x: (M, Kd) fp32 CUDA tensor (any row stride that is a multiple of 4); W: (Kd, N).
    fused=True writes one (M, 3N) tensor whose column blocks are Q, K and V and
    returns (qkv, q_view, k_view, v_view); otherwise returns three (M, N) tensors."""
    import torch
    M, Kd = x.shape
    N = wq.shape[1]
    if fused:
        qkv = torch.empty((M, 3 * N), dtype=torch.float32, device=x.device) if out is None else out
        outs = (qkv[:, :N], qkv[:, N:2 * N], qkv[:, 2 * N:])
    else:
        outs = tuple(torch.empty((M, N), dtype=torch.float32, device=x.device) for _ in range(3)) \
            if out is None else out
    shape = QKVShape(M, Kd, N, x.stride(0), outs[0].stride(0))

    def ptr(t):
        return t.data_ptr() if t is not None else None
    ws_ptr, ws_bytes = (None, 0)
    if workspace is not None:
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    check(lib.attn_qkv_proj_ex(ctypes.byref(shape), x.data_ptr(), wq.data_ptr(), wk.data_ptr(), wv.data_ptr(),
                               ptr(bq), ptr(bk), ptr(bv), outs[0].data_ptr(), outs[1].data_ptr(),
                               outs[2].data_ptr(), ws_ptr, ws_bytes, _stream()))
    return (qkv,) + outs if fused else outs


def decode_t(q, kcache, vcache, lens, heads: int, cap: int, max_len: int, kscale=None, vscale=None,
             out=None, workspace=None):
    """q: (n_seq, H*d) fp32; caches: (n_seq*cap, row_stride) fp32 or int8."""
    import torch
    n_seq, width = q.shape
    d = width // heads
    kv = I8 if kcache.dtype == torch.int8 else F32
    shape = DecodeShape(n_seq, heads, d, kv, kcache.stride(0), cap, max_len)
    out = torch.empty_like(q) if out is None else out
    ws_ptr, ws_bytes = (None, 0)
    if workspace is not None:
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    decode_ex(shape, q.data_ptr(), kcache.data_ptr(), vcache.data_ptr(),
              kscale.data_ptr() if kscale is not None else None,
              vscale.data_ptr() if vscale is not None else None,
              lens.data_ptr() if lens is not None else None, out.data_ptr(), ws_ptr, ws_bytes, _stream())
    return out


def quantize_int8_t(x, heads: int):
    """x: (rows, H*d) fp32 CUDA tensor -> (codes int8 same layout, scales (rows, H) fp32)."""
    import torch
    rows, width = x.shape
    d = width // heads
    codes = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    scales = torch.empty((rows, heads), dtype=torch.float32, device=x.device)
    check(lib.attn_kv_quantize_int8(x.data_ptr(), rows, heads, d, x.stride(0), codes.data_ptr(),
                                    scales.data_ptr(), _stream()))
    return codes, scales


def gather_permute_t(staging, world, batch, seq_len, heads, head_dim):
    import torch
    out = torch.empty((batch * seq_len, heads * head_dim), dtype=staging.dtype, device=staging.device)
    check(lib.attn_gather_permute(staging.data_ptr(), out.data_ptr(), world, batch, seq_len, heads, head_dim,
                                  _dtype_code(staging), _stream()))
    return out
