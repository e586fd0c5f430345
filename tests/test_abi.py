"""The C-ABI library loads here (no GPU), exports every symbol that
include/attn_b200.h declares, and its host-only logic behaves."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT

import attn_b200 as A


def declared_functions():
    src = open(os.path.join(ROOT, "include", "attn_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*ATTN_API\s+(?:const\s+)?[a-z_0-9]+\s*\*?\s*(attn_[a-z_0-9]+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_drop_in_surface():
    names = declared_functions()
    for must in ("attn_fwd", "attn_bwd", "attn_fwd_ex", "attn_bwd_ex", "attn_decode_ex",
                 "attn_cached_attention", "attn_kv_quantize_int8"):
        assert must in names


def test_every_declared_symbol_is_exported_and_bound():
    for name in declared_functions():
        assert hasattr(A.lib, name), f"{name} missing from libattn_b200.so"
        assert name in A.SIGNATURES, f"{name} has no ctypes signature in attn_b200.py"


def test_version_and_error_text():
    assert A.lib.attn_version() >= 1
    assert isinstance(A.last_error(), str)


def test_shard_range_partitions_exactly():
    for n, world in [(128, 1), (128, 8), (64, 3), (5, 8), (0, 2)]:
        spans = [A.shard_range(n, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        for (b0, e0), (b1, e1) in zip(spans, spans[1:]):
            assert e0 == b1
        sizes = [e - b for b, e in spans]
        assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    with pytest.raises(A.AttnError):
        A.shard_range(10, 2, 2)


def test_shard_lpt_balances_ragged_lengths():
    import synth
    lens = synth.uniform_int(7, 64, 1, 8192)
    ranks, load = A.shard_lpt(lens, 16, 8)
    assert ranks.shape == (64 * 16,) and set(ranks.tolist()) <= set(range(8))
    # recompute loads from the assignment
    per = np.zeros(8, np.int64)
    for u, r in enumerate(ranks):
        per[r] += lens[u // 16]
    assert np.array_equal(per, load)
    assert per.sum() == lens.sum() * 16
    # LPT bound: max load <= 4/3 of optimum (>= mean)
    assert per.max() <= per.mean() * 4 / 3 + lens.max()


def test_argument_validation_needs_no_gpu():
    s = A.Shape(1, 1, 8, 48, 0, 0)                       # unsupported head_dim
    assert A.lib.attn_fwd_ex(ctypes.byref(s), A.F32, 16, 16, 16, 16, None, None) == A.ERR_UNSUPPORTED
    assert "head_dim" in A.last_error()
    s = A.Shape(1, 2, 8, 64, 100, 0)                     # stride < H*d
    assert A.lib.attn_fwd_ex(ctypes.byref(s), A.F32, 16, 16, 16, 16, None, None) == A.ERR_INVALID
    s = A.Shape(1, 2, 8, 64, 0, 0)
    assert A.lib.attn_fwd_ex(ctypes.byref(s), 7, 16, 16, 16, 16, None, None) == A.ERR_UNSUPPORTED
    assert A.lib.attn_set_macro_shape(4, 12, 64, 128) == A.ERR_UNSUPPORTED   # T < d+1
    ds = A.DecodeShape(1, 16, 32, A.F32, 0, 10, 20)     # cap < max_len
    assert A.lib.attn_decode_ex(ctypes.byref(ds), 16, 16, 16, None, None, None, 16, None, 0, None) == A.ERR_INVALID
    ds = A.DecodeShape(1, 16, 32, A.I8, 0, 64, 64)      # int8 without scales
    assert A.lib.attn_decode_ex(ctypes.byref(ds), 16, 16, 16, None, None, None, 16, None, 0, None) == A.ERR_INVALID


def test_workspace_sizes():
    s = A.Shape(4, 16, 4096, 64, 0, 0)
    assert A.bwd_workspace_bytes(s, A.F32) >= 2 * 4 * 16 * 4096 * 4
    ds = A.DecodeShape(64, 16, 64, A.F32, 0, 8192, 8192)
    assert A.decode_workspace_bytes(ds) > 64 * 16 * 4


def test_drop_in_probs_buffer_is_large_enough_at_reference_shape():
    # gpu_kernels.h: B=4, H=12, T=1024, d=128; probs holds lse + a copy of att
    B, H, T, d = 4, 12, 1024, 128
    assert B * H * T * T >= B * H * T + B * T * H * d
    assert A.lib.attn_set_macro_shape(B, H, T, d) == A.OK


def test_probs_mode_validation_needs_no_gpu():
    assert A.lib.attn_set_probs_mode(5) == A.ERR_INVALID
    assert A.lib.attn_set_probs_mode(A.PROBS_LSE) == A.OK
    try:
        # probs holds only the log-sum-exp, so T < d+1 is allowed
        assert A.lib.attn_set_macro_shape(4, 12, 64, 128) == A.OK
    finally:
        assert A.lib.attn_set_probs_mode(A.PROBS_LSE_OUT) == A.OK
        assert A.lib.attn_set_macro_shape(4, 12, 1024, 128) == A.OK


def test_lse_mode_backward_of_an_unfilled_probs_buffer_exits():
    """attn_bwd in ATTN_PROBS_LSE mode with a `probs` that no attn_fwd filled
    stops with the drop-ins' CUDA_CHECK-style exit(1) before any device call."""
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r); import attn_b200 as A; "
            "A.lib.attn_set_probs_mode(A.PROBS_LSE); "
            "A.lib.attn_bwd(16, 16, 16, 16, 16, 16, 16, 16, 4096)") % os.path.dirname(A.__file__)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert r.returncode == 1
    assert "no attn_fwd has filled this `probs` buffer" in r.stderr


def test_qkv_proj_rejects_bad_arguments():
    """Argument checks of the fused QKV projection run before any CUDA call."""
    P16 = 1 << 20                                   # a 16-byte-aligned stand-in address
    ptrs = [P16] * 4
    outs = [P16] * 3
    assert A.lib.attn_qkv_proj_ex(None, *ptrs, None, None, None, *outs, None, 0, None) == A.ERR_INVALID
    bad = A.QKVShape(64, 96, 66, 0, 0)               # out_features not a multiple of 4
    assert A.lib.attn_qkv_proj_ex(ctypes.byref(bad), *ptrs, None, None, None, *outs, None, 0, None) == A.ERR_INVALID
    bad = A.QKVShape(64, 96, 64, 90, 0)              # X row stride shorter than its rows
    assert A.lib.attn_qkv_proj_ex(ctypes.byref(bad), *ptrs, None, None, None, *outs, None, 0, None) == A.ERR_INVALID
    ok = A.QKVShape(64, 96, 64, 0, 0)
    st = A.lib.attn_qkv_proj_ex(ctypes.byref(ok), P16 + 4, P16, P16, P16, None, None, None, *outs, None, 0, None)
    assert st == A.ERR_INVALID and "aligned" in A.last_error()
    st = A.lib.attn_qkv_proj_ex(ctypes.byref(ok), P16, None, P16, P16, None, None, None, *outs, None, 0, None)
    assert st == A.ERR_INVALID
    empty = A.QKVShape(0, 96, 64, 0, 0)              # no rows: nothing to do
    assert A.lib.attn_qkv_proj_ex(ctypes.byref(empty), *ptrs, None, None, None, *outs, None, 0, None) == A.OK


def test_qkv_workspace_size_and_check():
    shape = A.QKVShape(4096, 1536, 1536, 0, 0)
    assert A.lib.attn_qkv_workspace_bytes(ctypes.byref(shape)) == 2 * 3 * 1536 * 1536 * 4
    odd = A.QKVShape(10, 37, 12, 40, 0)            # in_features rounded up to 4 in the split weights
    assert A.lib.attn_qkv_workspace_bytes(ctypes.byref(odd)) == 2 * ((3 * 12 * 40 * 4 + 255) // 256 * 256)
    P16 = 1 << 20
    st = A.lib.attn_qkv_proj_ex(ctypes.byref(shape), P16, P16, P16, P16, None, None, None, P16, P16, P16,
                                P16, 1024, None)   # a caller workspace that is too small
    assert st == A.ERR_WORKSPACE


def test_bwd_tc_workspace_size():
    """The optional workspace for the tensor-core backward at d 96 / 128."""
    tr = A.Shape(4, 12, 1024, 128, 0, 0)
    big = A.lib.attn_bwd_tc_workspace_bytes(ctypes.byref(tr))
    floats = 2 * 48 * 1024 * (1024 + 5 * 128 + 1) + 48 * 1024 * 1024
    assert floats * 4 <= big < floats * 4 + 16 * 256
    for shape in (A.Shape(4, 12, 1024, 64, 0, 0), A.Shape(1, 2, 130, 128, 0, 0), A.Shape(1, 2, 128, 32, 0, 0)):
        assert A.lib.attn_bwd_tc_workspace_bytes(ctypes.byref(shape)) == 0     # d 64 / 32, or T % 4 != 0
