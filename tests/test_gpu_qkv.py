"""The fused QKV projection (attn_qkv_proj_ex / attn_qkv_proj) against the
oracle's restatement of train.c's matmul_forward (train.c:181-211), the
fixtures the reference's own matmul_forward produced, and -- at the reference
GPU trainer's shape -- an fp32 cuBLAS SGEMM, the arithmetic of gemm_nn
(gpu_kernels.cu:112-120) that train_kaggle.cu:152-154 calls three times.
Tolerance: 1e-5 of max|ref| (fp32 arithmetic)."""
import ctypes
import os

import numpy as np
import pytest

from conftest import ROOT, golden, rel_err
from oracle import oracle as O
import synth

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5


@pytest.fixture(scope="module")
def A(cuda):
    import attn_b200
    return attn_b200


def dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


def case(seed, M, K, N, w_std=0.02, x_std=1.0):
    x = synth.normal(seed, (M, K), 0, x_std)
    ws = [synth.normal(seed + 1 + i, (K, N), 0, w_std) for i in range(3)]
    bs = [synth.normal(seed + 4 + i, (N,), 0, 0.1) for i in range(3)]
    return x, ws, bs


@pytest.mark.parametrize("name", ["qkv_m72_k96_n64", "qkv_m37_k52_n36"])
def test_qkv_golden(A, name):
    z = golden(name)
    outs = A.qkv_proj_t(dev(z["x"]), dev(z["wq"]), dev(z["wk"]), dev(z["wv"]), dev(z["bq"]), dev(z["bk"]),
                        dev(z["bv"]))
    for out, want in zip(outs, (z["q"], z["k"], z["v"])):
        assert rel_err(out.cpu().numpy(), want) < F32_TOL


# ragged edges: rows, columns and k not multiples of the 128 x 128 x 32 tiles
@pytest.mark.parametrize("M,K,N", [(128, 256, 128), (200, 100, 68), (1, 4, 4), (333, 1000, 260), (1024, 512, 512)])
@pytest.mark.parametrize("with_bias", [True, False])
def test_qkv_vs_oracle(A, M, K, N, with_bias):
    x, ws, bs = case(7 * M + K, M, K, N)
    if not with_bias:
        bs = [None] * 3
    outs = A.qkv_proj_t(dev(x), *(dev(w) for w in ws), *(dev(b) if b is not None else None for b in bs))
    for out, want in zip(outs, O.qkv_proj(x, ws, bs, f64=True)):
        assert rel_err(out.cpu().numpy(), want) < F32_TOL


def test_qkv_fused_layout_strided_input(A):
    """X read with a row stride (a column block of a wider tensor), Q, K, V
    written as the three column blocks of one (M, 3N) tensor -- the layout the
    attention kernels read with in_row_stride = 3N; the attention over it
    matches the attention over separate tensors."""
    import torch
    M, K, N, B, H = 256, 192, 128, 2, 2
    x, ws, bs = case(31, M, K, N)
    wide = torch.zeros((M, K + 64), dtype=torch.float32, device="cuda")
    wide[:, 32:32 + K] = dev(x)
    xs = wide[:, 32:32 + K]
    qkv, q, k, v = A.qkv_proj_t(xs, *(dev(w) for w in ws), *(dev(b) for b in bs), fused=True)
    assert q.stride(0) == 3 * N
    for out, want in zip((q, k, v), O.qkv_proj(x, ws, bs, f64=True)):
        assert rel_err(out.cpu().numpy(), want) < F32_TOL
    o_fused, _ = A.forward_t(q, k, v, H, B)
    o_sep, _ = A.forward_t(q.contiguous(), k.contiguous(), v.contiguous(), H, B)
    assert torch.equal(o_fused, o_sep)


def test_qkv_positive_sums_do_not_drift(A):
    """All-positive operands over a long k range: the tensor core's TMEM
    accumulation is not round-to-nearest, so the kernel restarts its TMEM sums
    every 256 k and adds them in fp32; a drift would show here first."""
    M, K, N = 256, 4096, 128
    x = np.abs(synth.normal(41, (M, K)))
    ws = [np.abs(synth.normal(42 + i, (K, N), 0, 0.02)) for i in range(3)]
    outs = A.qkv_proj_t(dev(x), *(dev(w) for w in ws))
    for out, want in zip(outs, O.qkv_proj(x, ws, f64=True)):
        assert rel_err(out.cpu().numpy(), want) < F32_TOL


def test_qkv_trainer_shape_vs_cublas_sgemm(A):
    """The reference GPU trainer's own shape (M = B*T = 4096, DIM 1536,
    gpu_kernels.h:17-31) against fp32 cuBLAS SGEMM + bias (gemm_nn's
    arithmetic), whole tensors, and sampled rows against the fp64 oracle."""
    import torch
    M, K, N = 4096, 1536, 1536
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn((M, K), generator=g, device="cuda")
    ws = [torch.randn((K, N), generator=g, device="cuda") * 0.02 for _ in range(3)]
    bs = [torch.randn((N,), generator=g, device="cuda") * 0.1 for _ in range(3)]
    outs = A.qkv_proj_t(x, *ws, *bs)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        refs = [x @ w + b for w, b in zip(ws, bs)]
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    rows = np.arange(0, M, 97)
    xs = x[rows].cpu().numpy()
    for out, ref, w, b in zip(outs, refs, ws, bs):
        assert rel_err(out.cpu().numpy(), ref.cpu().numpy()) < F32_TOL
        want = O.matmul_forward(xs, w.cpu().numpy(), b.cpu().numpy(), f64=True)
        assert rel_err(out[rows].cpu().numpy(), want) < F32_TOL
    # the reference's own gemm_nn, built from gpu_kernels.cu into baseline/_ref/
    path = os.path.join(ROOT, "baseline", "_ref", "libref_gpu_4x12x1024x128.so")
    if os.path.exists(path):
        L = ctypes.CDLL(path)
        L.refgpu_gemm_nn.restype = None
        L.refgpu_init()
        P, I = ctypes.c_void_p, ctypes.c_int
        torch.cuda.synchronize()
        for out, w, b in zip(outs, ws, bs):
            theirs = torch.empty_like(out)
            L.refgpu_gemm_nn(P(x.data_ptr()), P(w.data_ptr()), P(b.data_ptr()), P(theirs.data_ptr()),
                             I(M), I(K), I(N))
            torch.cuda.synchronize()
            assert rel_err(out.cpu().numpy(), theirs.cpu().numpy()) < F32_TOL


def test_qkv_dropin_signature_and_repeat(A):
    """attn_qkv_proj (gemm_nn's argument style, default stream) equals the _ex
    entry point bit for bit, call after call (deterministic), with the
    library's workspace or the caller's."""
    import torch
    M, K, N = 300, 256, 192
    x, ws, bs = case(77, M, K, N)
    xd, wd, bd = dev(x), [dev(w) for w in ws], [dev(b) for b in bs]
    ref = A.qkv_proj_t(xd, *wd, *bd)
    torch.cuda.synchronize()
    for _ in range(2):
        outs = [torch.full((M, N), float("nan"), device="cuda") for _ in range(3)]
        A.lib.attn_qkv_proj(xd.data_ptr(), *(w.data_ptr() for w in wd), *(b.data_ptr() for b in bd),
                            *(o.data_ptr() for o in outs), M, K, N)
        torch.cuda.synchronize()
        for o, r in zip(outs, ref):
            assert torch.equal(o, r)
    # a caller workspace instead of the library's own gives the same bits
    shape = A.QKVShape(M, K, N, 0, 0)
    ws = torch.empty(A.lib.attn_qkv_workspace_bytes(ctypes.byref(shape)), dtype=torch.uint8, device="cuda")
    mine = A.qkv_proj_t(xd, *wd, *bd, workspace=ws)
    for o, r in zip(mine, ref):
        assert torch.equal(o, r)
    code = ctypes.c_int(0)
    A.check(A.lib.attn_device_error(0, ctypes.byref(code)))
    assert code.value == 0


def test_qkv_bounded_wait_timeout_path(A):
    """Failure detection in a TMEM-holding tensor-core kernel without a fault:
    a test hook makes the QKV kernel's MMA warp wait on a barrier nothing
    arrives at.  The bounded wait runs out, the kernel records 0x5ff in the
    device error word, every role stops, and the teardown frees TMEM -- the
    next call allocates TMEM on every SM again, is correct and leaves the
    error word clear."""
    import torch
    M, K, N = 512, 256, 128
    x, ws, bs = case(91, M, K, N)
    xd, wd, bd = dev(x), [dev(w) for w in ws], [dev(b) for b in bs]
    code = ctypes.c_int()
    A.check(A.lib.attn_device_error(0, ctypes.byref(code)))       # clear
    A.check(A.lib.attn_debug_qkv_timeout(1, 200000))
    try:
        A.qkv_proj_t(xd, *wd, *bd)
        torch.cuda.synchronize()
    finally:
        A.check(A.lib.attn_debug_qkv_timeout(0, 0))                 # disarmed whatever ran
    A.check(A.lib.attn_device_error(0, ctypes.byref(code)))
    assert code.value == 0x5ff
    outs = A.qkv_proj_t(xd, *wd, *bd)
    torch.cuda.synchronize()
    A.check(A.lib.attn_device_error(0, ctypes.byref(code)))
    assert code.value == 0
    for out, want in zip(outs, O.qkv_proj(x, ws, bs, f64=True)):
        assert rel_err(out.cpu().numpy(), want) < F32_TOL
