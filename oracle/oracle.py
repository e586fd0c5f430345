"""ctypes wrappers of the parity checker (TEST INFRASTRUCTURE ONLY).

liboracle.so is the C restatement in attn_oracle.c; oracle/_ref/*.so are the
reference's own attention routines compiled from its unmodified sources (see
oracle/Makefile).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline may use this module; the product never does.
"""
import ctypes
import glob
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_F = ctypes.POINTER(ctypes.c_float)
_lib = None


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise ImportError(f"{path} not built; run `make -C oracle`")
        _lib = ctypes.CDLL(path)
        V, I, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_long
        _lib.oracle_attn_forward.argtypes = [V, V, V, V, V, V, I, I, I, I, L]
        _lib.oracle_attn_forward_f64.argtypes = [V, V, V, V, I, I, I, I, L]
        _lib.oracle_attn_backward.argtypes = [V, V, V, V, V, V, V, V, I, I, I, I, L]
        _lib.oracle_cached_attention.argtypes = [V, V, V, V, I, I, I, L]
        _lib.oracle_cached_attention_f64.argtypes = [V, V, V, V, I, I, I, L]
        _lib.oracle_quantize_kv_int8.argtypes = [V, V, V, L, I, I, L]
        _lib.oracle_dequantize_kv_int8.argtypes = [V, V, V, L, I, I, L]
        _lib.oracle_matmul_forward.argtypes = [V, V, V, V, I, I, I, L]
        _lib.oracle_matmul_forward_f64.argtypes = [V, V, V, V, I, I, I, L]
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------------------
# C restatement
# ---------------------------------------------------------------------------
def attn_forward(q, k, v, B, T, H, d, want_probs=False, want_lse=True):
    q, k, v = _f32(q), _f32(k), _f32(v)
    att = np.zeros((B * T, H * d), np.float32)
    probs = np.zeros((B * H, T, T), np.float32) if want_probs else None
    lse = np.zeros((B, H, T), np.float32) if want_lse else None
    lib().oracle_attn_forward(_p(q), _p(k), _p(v), _p(att), _p(probs), _p(lse), B, T, H, d, H * d)
    return att, probs, lse


def attn_forward_f64(q, k, v, B, T, H, d):
    q, k, v = _f32(q), _f32(k), _f32(v)
    att = np.zeros((B * T, H * d), np.float32)
    lib().oracle_attn_forward_f64(_p(q), _p(k), _p(v), _p(att), B, T, H, d, H * d)
    return att


def attn_backward(do, q, k, v, probs, B, T, H, d):
    """Gradients from zero (train.c accumulates into zeroed buffers)."""
    do, q, k, v, probs = _f32(do), _f32(q), _f32(k), _f32(v), _f32(probs)
    dq = np.zeros_like(q)
    dk = np.zeros_like(q)
    dv = np.zeros_like(q)
    lib().oracle_attn_backward(_p(dq), _p(dk), _p(dv), _p(do), _p(q), _p(k), _p(v), _p(probs), B, T, H, d, H * d)
    return dq, dk, dv


def cached_attention(q, kcache, vcache, pos, H, d, row_stride=None, f64=False):
    q, kcache, vcache = _f32(q), _f32(kcache), _f32(vcache)
    rs = row_stride or H * d
    out = np.zeros(H * d, np.float32)
    fn = lib().oracle_cached_attention_f64 if f64 else lib().oracle_cached_attention
    fn(_p(q), _p(kcache), _p(vcache), _p(out), pos, H, d, rs)
    return out


def quantize_kv_int8(x, H, d):
    x = _f32(x)
    rows = x.shape[0]
    codes = np.zeros(x.shape, np.int8)
    scales = np.zeros((rows, H), np.float32)
    lib().oracle_quantize_kv_int8(_p(x), _p(codes), _p(scales), rows, H, d, x.shape[1])
    return codes, scales


def dequantize_kv_int8(codes, scales, H, d):
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = _f32(scales)
    x = np.zeros(codes.shape, np.float32)
    lib().oracle_dequantize_kv_int8(_p(codes), _p(scales), _p(x), codes.shape[0], H, d, codes.shape[1])
    return x


def lse_to_probs(q, k, lse, B, T, H, d):
    """Rebuild the reference's probs matrix from lse (numpy, small shapes)."""
    qh = q.reshape(B, T, H, d).transpose(0, 2, 1, 3).astype(np.float64)
    kh = k.reshape(B, T, H, d).transpose(0, 2, 1, 3).astype(np.float64)
    s = qh @ kh.transpose(0, 1, 3, 2) / np.sqrt(d)
    p = np.exp(s - lse.reshape(B, H, T, 1).astype(np.float64))
    p = np.tril(p)
    return p.reshape(B * H, T, T).astype(np.float32)


def matmul_forward(x, w, bias=None, f64=False):
    """x (M, K) @ w (K, N) + bias: train.c:181-211 restated (fp32, or fp64 sums)."""
    x, w = _f32(x), _f32(w)
    b = _f32(bias) if bias is not None else None
    M, K = x.shape
    N = w.shape[1]
    out = np.zeros((M, N), np.float64 if f64 else np.float32)
    fn = lib().oracle_matmul_forward_f64 if f64 else lib().oracle_matmul_forward
    fn(_p(out), _p(x), _p(w), _p(b), M, K, N, K)
    return out


def qkv_proj(x, ws, bs=(None, None, None), f64=False):
    """The three projections of train.c:517-519 / train_kaggle.cu:152-154."""
    return tuple(matmul_forward(x, w, b, f64) for w, b in zip(ws, bs))


# ---------------------------------------------------------------------------
# the reference itself, compiled from its sources
# ---------------------------------------------------------------------------
_ref_cache = {}


def ref_available():
    return bool(glob.glob(os.path.join(REF_DIR, "libref_*.so")))


def _ref(name):
    if name not in _ref_cache:
        path = os.path.join(REF_DIR, name)
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (needs the reference sources; see oracle/Makefile)")
        L = ctypes.CDLL(path)
        V, I = ctypes.c_void_p, ctypes.c_int
        if name.startswith("libref_train"):
            L.ref_attention_forward.argtypes = [V, V, V, V, V, I, I]
            L.ref_attention_backward.argtypes = [V, V, V, V, V, V, V, V, I, I]
            L.ref_matmul_forward.argtypes = [V, V, V, V, I, I, I]
        elif name.startswith("libref_quant"):
            L.ref_quantize_A.argtypes = [V, V, I, I, I]
            L.ref_quantize_A.restype = ctypes.c_float
        else:
            L.ref_cached_attention.argtypes = [V, V, V, V, V, I]
            L.ref_multihead_attention.argtypes = [V, V, V, V, V, I]
        _ref_cache[name] = L
    return _ref_cache[name]


def ref_train_name(H, d):
    return f"libref_train_h{H}_d{d}.so"


def ref_decode_name(H, d, t_max):
    return f"libref_decode_h{H}_d{d}_t{t_max}.so"


def ref_attention_forward(q, k, v, B, T, H, d):
    L = _ref(ref_train_name(H, d))
    q, k, v = _f32(q), _f32(k), _f32(v)
    att = np.zeros((B * T, H * d), np.float32)
    probs = np.zeros((B * H, T, T), np.float32)
    L.ref_attention_forward(_p(q), _p(k), _p(v), _p(att), _p(probs), B, T)
    return att, probs


def ref_attention_backward(do, q, k, v, probs, B, T, H, d):
    L = _ref(ref_train_name(H, d))
    do, q, k, v, probs = _f32(do), _f32(q), _f32(k), _f32(v), _f32(probs)
    dq, dk, dv = np.zeros_like(q), np.zeros_like(q), np.zeros_like(q)
    L.ref_attention_backward(_p(dq), _p(dk), _p(dv), _p(do), _p(q), _p(k), _p(v), _p(probs), B, T)
    return dq, dk, dv


def ref_quantize_kv_int8(x, H, d):
    """The reference's quantize_A (gemm_bench.c:225-236) applied to every
    (row, head) slice: returns signed codes (its u8 output minus the +128
    offset) and the per-slice scales."""
    L = _ref("libref_quant.so")
    x = _f32(x)
    rows = x.shape[0]
    codes = np.zeros(x.shape, np.int8)
    scales = np.zeros((rows, H), np.float32)
    buf = np.zeros(d, np.uint8)
    for r in range(rows):
        for h in range(H):
            sl = np.ascontiguousarray(x[r, h * d:(h + 1) * d])
            scales[r, h] = L.ref_quantize_A(_p(sl), _p(buf), 1, d, d)
            codes[r, h * d:(h + 1) * d] = (buf.astype(np.int16) - 128).astype(np.int8)
    return codes, scales


def ref_cached_attention(q, kcache, vcache, pos, H, d, t_max):
    """kcache/vcache: (t_max, H*d) slabs as in KVCache (model.h:42-45)."""
    L = _ref(ref_decode_name(H, d, t_max))
    q, kcache, vcache = _f32(q), _f32(kcache), _f32(vcache)
    out = np.zeros(H * d, np.float32)
    scores = np.zeros(H * t_max, np.float32)
    L.ref_cached_attention(_p(q), _p(kcache), _p(vcache), _p(out), _p(scores), pos)
    return out


def ref_matmul_forward(x, w, bias=None):
    """The reference's own matmul_forward (train.c:181-211), any shape (it is
    shape-independent; the object of the smallest training build is used)."""
    L = _ref(ref_train_name(1, 64))
    x, w = _f32(x), _f32(w)
    b = _f32(bias) if bias is not None else None
    M, K = x.shape
    N = w.shape[1]
    out = np.zeros((M, N), np.float32)
    L.ref_matmul_forward(_p(out), _p(x), _p(w), _p(b), M, K, N)
    return out
