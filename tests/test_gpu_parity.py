"""CUDA path vs the oracle and the reference-generated fixtures, through the
C ABI.  Tolerances (max|out-ref| / max|ref|): 1e-5 for fp32 arithmetic and
for attention over a dequantised INT8 cache; 2e-2 (forward) and 3e-2
(backward) for bf16 tensor-core products against fp32 over the same
bf16-rounded inputs; bit-exact for the INT8 quantiser."""
import ctypes

import numpy as np
import pytest

from conftest import golden, rel_err
from oracle import oracle as O
import synth

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
BF16_FWD_TOL = 2e-2
BF16_BWD_TOL = 3e-2


@pytest.fixture(scope="module")
def A(cuda):
    import attn_b200
    return attn_b200


def dev(x, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t.to(dtype) if dtype is not None else t


def host(t):
    import torch
    return t.float().cpu().numpy() if t.dtype == torch.bfloat16 else t.cpu().numpy()


def bf16_round(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).float().numpy()


def qkv(seed, B, T, H, d, std=0.5):
    return (synth.normal(seed, (B * T, H * d), 0, std), synth.normal(seed + 1, (B * T, H * d), 0, std),
            synth.normal(seed + 2, (B * T, H * d), 0, std))


# ---------------------------------------------------------------------------
# forward
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["fwd_h4_d32", "fwd_h2_d64", "fwd_h2_d128", "fwd_h2_d96", "fwd_t1"])
def test_forward_f32_golden(A, name):
    z = golden(name)
    B, T, H, d = (int(x) for x in z["shape"])
    out, lse = A.forward_t(dev(z["q"]), dev(z["k"]), dev(z["v"]), H, B)
    assert rel_err(host(out), z["att"]) < F32_TOL
    probs = O.lse_to_probs(z["q"], z["k"], host(lse).reshape(B, H, T), B, T, H, d)
    assert rel_err(probs, z["probs"]) < F32_TOL


@pytest.mark.parametrize("B,T,H,d", [(2, 130, 3, 32), (1, 200, 2, 64), (1, 77, 2, 96), (1, 129, 2, 128),
                                     (1, 64, 1, 64), (3, 1, 2, 32), (1, 256, 4, 64), (2, 300, 3, 128),
                                     (1, 515, 2, 96), (2, 1, 1, 128), (1, 33, 1, 96)])
def test_forward_f32_vs_oracle(A, B, T, H, d):
    q, k, v = qkv(11 * T + d, B, T, H, d)
    ref, _, rlse = O.attn_forward(q, k, v, B, T, H, d)
    out, lse = A.forward_t(dev(q), dev(k), dev(v), H, B)
    assert rel_err(host(out), ref) < F32_TOL
    assert rel_err(host(lse), rlse.reshape(-1)) < F32_TOL


@pytest.mark.parametrize("B,T,H,d", [(2, 130, 3, 32), (1, 300, 2, 64), (1, 129, 2, 128), (2, 1024, 2, 64),
                                     (1, 77, 2, 96), (1, 5, 1, 64)])
def test_forward_bf16_vs_fp32_oracle(A, B, T, H, d):
    import torch
    q, k, v = (bf16_round(x) for x in qkv(7 * T + d, B, T, H, d))
    ref, _, rlse = O.attn_forward(q, k, v, B, T, H, d)
    out, lse = A.forward_t(dev(q, torch.bfloat16), dev(k, torch.bfloat16), dev(v, torch.bfloat16), H, B)
    assert out.dtype == torch.bfloat16
    assert rel_err(host(out), ref) < BF16_FWD_TOL
    assert np.abs(host(lse) - rlse.reshape(-1)).max() < 0.05


def test_forward_strided_heads_subset(A):
    """A call may cover a head slice of wider rows (the per-rank shard of a
    multi-GPU split): in/out strides larger than H*d."""
    import torch
    B, T, H, d = 2, 96, 4, 64
    q, k, v = qkv(5, B, T, H, d)
    ref, _, _ = O.attn_forward(q, k, v, B, T, H, d)
    qd, kd, vd = dev(q), dev(k), dev(v)
    h0, hn = 1, 2
    out = torch.zeros((B * T, hn * d), device="cuda")
    shape = A.Shape(B, hn, T, d, H * d, hn * d)
    A.fwd_ex(shape, A.F32, qd[:, h0 * d:].data_ptr(), kd[:, h0 * d:].data_ptr(), vd[:, h0 * d:].data_ptr(),
             out.data_ptr(), None)
    torch.cuda.synchronize()
    assert rel_err(host(out), ref[:, h0 * d:(h0 + hn) * d]) < F32_TOL


@pytest.mark.parametrize("dt,d", [("f32", 64), ("bf16", 64), ("f32", 128)])
def test_fused_qkv_layout(A, dt, d):
    """Q, K and V as the three column blocks of one (B*T, 3*H*d) projection
    output (a fused Wq|Wk|Wv GEMM), and dQ, dK, dV written into the column
    blocks of one gradient tensor of that width: the kernels take the row
    stride through their tensor maps, so no head-major copy is needed."""
    import torch
    B, T, H = 2, 200, 3
    q, k, v = qkv(31, B, T, H, d)
    do = synth.normal(32, (B * T, H * d))
    tdt, code = (torch.float32, A.F32) if dt == "f32" else (torch.bfloat16, A.BF16)
    ftol, btol = (F32_TOL, F32_TOL) if dt == "f32" else (BF16_FWD_TOL, BF16_BWD_TOL)
    if dt == "bf16":
        q, k, v, do = (bf16_round(x) for x in (q, k, v, do))
    ref, probs, _ = O.attn_forward(q, k, v, B, T, H, d, want_probs=True)
    rq, rk, rv = O.attn_backward(do, q, k, v, probs, B, T, H, d)
    W = 3 * H * d
    qkv_d = torch.cat([torch.as_tensor(x, device="cuda") for x in (q, k, v)], dim=1).to(tdt).contiguous()
    o_d = torch.zeros((B * T, W), dtype=tdt, device="cuda")
    g_d = torch.zeros((B * T, W), dtype=tdt, device="cuda")
    g_d[:, :H * d] = torch.as_tensor(do, device="cuda").to(tdt)
    lse = torch.zeros(B * H * T, device="cuda")
    shape = A.Shape(B, H, T, d, W, W)
    col = lambda t, i: t[:, i * H * d:].data_ptr()          # noqa: E731
    A.fwd_ex(shape, code, col(qkv_d, 0), col(qkv_d, 1), col(qkv_d, 2), col(o_d, 0), lse.data_ptr())
    dqkv = torch.full((B * T, W), 7.0, dtype=tdt, device="cuda")
    ws = torch.zeros(A.bwd_workspace_bytes(shape, code), dtype=torch.uint8, device="cuda")
    A.check(A.lib.attn_bwd_ex(ctypes.byref(shape), code, col(g_d, 0), col(qkv_d, 0), col(qkv_d, 1),
                              col(qkv_d, 2), col(o_d, 0), lse.data_ptr(), col(dqkv, 0), col(dqkv, 1),
                              col(dqkv, 2), 0, ws.data_ptr(), ws.numel(), None))
    torch.cuda.synchronize()
    h = lambda t, i: host(t[:, i * H * d:(i + 1) * H * d].float())   # noqa: E731
    assert rel_err(h(o_d, 0), ref) < ftol
    assert bool((o_d[:, H * d:] == 0).all())                 # only O's own columns are written
    for i, r in enumerate((rq, rk, rv)):
        assert rel_err(h(dqkv, i), r) < btol


def test_forward_deterministic(A):
    q, k, v = qkv(3, 2, 300, 2, 64)
    a, _ = A.forward_t(dev(q), dev(k), dev(v), 2, 2)
    b, _ = A.forward_t(dev(q), dev(k), dev(v), 2, 2)
    assert np.array_equal(host(a), host(b))


# ---------------------------------------------------------------------------
# backward
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["bwd_h2_d64", "bwd_h4_d32"])
def test_backward_f32_golden(A, name):
    z = golden(name)
    B, T, H, d = (int(x) for x in z["shape"])
    q, k, v, do = dev(z["q"]), dev(z["k"]), dev(z["v"]), dev(z["do"])
    o, lse = A.forward_t(q, k, v, H, B)
    dq, dk, dv = A.backward_t(do, q, k, v, o, lse, H, B)
    assert rel_err(host(dq), z["dq"]) < F32_TOL
    assert rel_err(host(dk), z["dk"]) < F32_TOL
    assert rel_err(host(dv), z["dv"]) < F32_TOL


def test_backward_accumulate_flag(A):
    """accumulate=1 adds into the gradients like train.c:372; 0 sets them
    like gpu_kernels.cu's attn_bwd (beta = 0)."""
    z = golden("bwd_h4_d32")
    B, T, H, d = (int(x) for x in z["shape"])
    q, k, v, do = dev(z["q"]), dev(z["k"]), dev(z["v"]), dev(z["do"])
    o, lse = A.forward_t(q, k, v, H, B)
    base = synth.normal(77, z["q"].shape)
    dq, dk, dv = dev(base), dev(base), dev(base)
    A.backward_t(do, q, k, v, o, lse, H, B, dq, dk, dv, accumulate=True)
    assert rel_err(host(dq), base + z["dq"]) < F32_TOL
    assert rel_err(host(dv), base + z["dv"]) < F32_TOL
    A.backward_t(do, q, k, v, o, lse, H, B, dq, dk, dv, accumulate=False)
    assert rel_err(host(dk), z["dk"]) < F32_TOL


@pytest.mark.parametrize("B,T,H,d", [(1, 200, 2, 64), (2, 70, 2, 32), (1, 129, 1, 128), (1, 100, 2, 96),
                                     (1, 1, 2, 64)])
def test_backward_f32_vs_oracle(A, B, T, H, d):
    q, k, v = qkv(13 * T + d, B, T, H, d)
    do = synth.normal(99 + T, (B * T, H * d))
    _, probs, _ = O.attn_forward(q, k, v, B, T, H, d, want_probs=True)
    rq, rk, rv = O.attn_backward(do, q, k, v, probs, B, T, H, d)
    qd, kd, vd, gd = dev(q), dev(k), dev(v), dev(do)
    o, lse = A.forward_t(qd, kd, vd, H, B)
    dq, dk, dv = A.backward_t(gd, qd, kd, vd, o, lse, H, B)
    assert rel_err(host(dq), rq) < F32_TOL
    assert rel_err(host(dk), rk) < F32_TOL
    assert rel_err(host(dv), rv) < F32_TOL


@pytest.mark.parametrize("B,T,H,d", [(1, 200, 2, 64), (2, 130, 2, 32), (1, 256, 1, 128)])
def test_backward_bf16_vs_fp32_oracle(A, B, T, H, d):
    import torch
    q, k, v = (bf16_round(x) for x in qkv(17 * T + d, B, T, H, d))
    do = bf16_round(synth.normal(5 + T, (B * T, H * d)))
    _, probs, _ = O.attn_forward(q, k, v, B, T, H, d, want_probs=True)
    rq, rk, rv = O.attn_backward(do, q, k, v, probs, B, T, H, d)
    bf = torch.bfloat16
    qd, kd, vd, gd = dev(q, bf), dev(k, bf), dev(v, bf), dev(do, bf)
    o, lse = A.forward_t(qd, kd, vd, H, B)
    dq, dk, dv = A.backward_t(gd, qd, kd, vd, o, lse, H, B)
    assert rel_err(host(dq), rq) < BF16_BWD_TOL
    assert rel_err(host(dk), rk) < BF16_BWD_TOL
    assert rel_err(host(dv), rv) < BF16_BWD_TOL


@pytest.mark.parametrize("dt,pad_in,pad_out", [("f32", 4, 8), ("bf16", 4, 12)])
def test_backward_padded_rows(A, dt, pad_in, pad_out):
    """Rows wider than H*d (strides a multiple of 4 elements, as the C ABI
    requires; at bf16 an input stride that is not a multiple of 8 keeps the
    call off the tensor-core kernels): the row statistics and the gradients
    read and write only the first H*d columns of each row."""
    import torch
    B, T, H, d = 1, 130, 2, 32
    q, k, v = qkv(23, B, T, H, d)
    do = synth.normal(24, (B * T, H * d))
    tdt, code, tol = (torch.float32, A.F32, F32_TOL) if dt == "f32" else (torch.bfloat16, A.BF16, BF16_BWD_TOL)
    if dt == "bf16":
        q, k, v, do = (bf16_round(x) for x in (q, k, v, do))
    _, probs, _ = O.attn_forward(q, k, v, B, T, H, d, want_probs=True)
    rq, rk, rv = O.attn_backward(do, q, k, v, probs, B, T, H, d)
    wi, wo = H * d + pad_in, H * d + pad_out

    def padded(x, w):
        t = torch.zeros((B * T, w), dtype=tdt, device="cuda")
        t[:, :H * d] = torch.as_tensor(x, device="cuda").to(tdt)
        return t

    qd, kd, vd, gd = (padded(x, wi) for x in (q, k, v, do))
    od = torch.zeros((B * T, wo), dtype=tdt, device="cuda")
    lse = torch.zeros(B * H * T, device="cuda")
    shape = A.Shape(B, H, T, d, wi, wo)
    A.fwd_ex(shape, code, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(), lse.data_ptr())
    grads = [torch.zeros((B * T, wo), dtype=tdt, device="cuda") for _ in range(3)]
    ws_bytes = A.bwd_workspace_bytes(shape, code)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    A.bwd_ex(shape, code, gd.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(), lse.data_ptr(),
             grads[0].data_ptr(), grads[1].data_ptr(), grads[2].data_ptr(), 0, ws.data_ptr(), ws_bytes)
    torch.cuda.synchronize()
    for g, r in zip(grads, (rq, rk, rv)):
        assert rel_err(host(g[:, :H * d]), r) < tol
        assert not (g[:, H * d:] != 0).any()     # the padding columns stay untouched


def test_backward_deterministic_and_workspace_check(A):
    import torch
    q, k, v = qkv(8, 1, 150, 2, 64)
    do = synth.normal(9, q.shape)
    qd, kd, vd, gd = dev(q), dev(k), dev(v), dev(do)
    o, lse = A.forward_t(qd, kd, vd, 2, 1)
    r1 = A.backward_t(gd, qd, kd, vd, o, lse, 2, 1)
    r2 = A.backward_t(gd, qd, kd, vd, o, lse, 2, 1)
    for a, b in zip(r1, r2):
        assert np.array_equal(host(a), host(b))
    shape = A.Shape(1, 2, 150, 64, 0, 0)
    small = torch.empty(64, dtype=torch.uint8, device="cuda")
    st = A.lib.attn_bwd_ex(ctypes.byref(shape), A.F32, gd.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(),
                           o.data_ptr(), lse.data_ptr(), r1[0].data_ptr(), r1[1].data_ptr(), r1[2].data_ptr(), 0,
                           small.data_ptr(), 64, None)
    assert st == A.ERR_WORKSPACE


# ---------------------------------------------------------------------------
# drop-in attn_fwd / attn_bwd (gpu_kernels.h:67-72)
# ---------------------------------------------------------------------------
def test_drop_in_fwd_bwd(A):
    import torch
    B, T, H, d = 2, 130, 2, 64
    A.check(A.lib.attn_set_macro_shape(B, H, T, d))
    try:
        q, k, v = qkv(21, B, T, H, d)
        do = synth.normal(22, q.shape)
        ref, probs, _ = O.attn_forward(q, k, v, B, T, H, d, want_probs=True)
        rq, rk, rv = O.attn_backward(do, q, k, v, probs, B, T, H, d)
        qd, kd, vd, gd = dev(q), dev(k), dev(v), dev(do)
        att = torch.empty_like(qd)
        probs_buf = torch.empty(B * H * T * T, device="cuda")
        scratch = torch.empty(B * H * T * T, device="cuda")
        dq, dk, dv = (torch.full_like(qd, 7.0) for _ in range(3))   # SET, not accumulated
        torch.cuda.synchronize()
        A.lib.attn_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), att.data_ptr(), probs_buf.data_ptr())
        A.lib.attn_bwd(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), scratch.data_ptr(), gd.data_ptr(),
                       qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), probs_buf.data_ptr())
        torch.cuda.synchronize()
        assert rel_err(host(att), ref) < F32_TOL
        assert rel_err(host(dq), rq) < F32_TOL
        assert rel_err(host(dk), rk) < F32_TOL
        assert rel_err(host(dv), rv) < F32_TOL
    finally:
        A.lib.attn_set_macro_shape(4, 12, 1024, 128)


@pytest.mark.parametrize("B,H,T,d", [(2, 2, 256, 128), (1, 2, 132, 128), (1, 3, 200, 96), (1, 1, 516, 128)])
def test_drop_in_bwd_on_tensor_cores(A, B, H, T, d):
    """The drop-in backward at d 96 / 128 in the default probs mode, every
    product on the tensor cores (3xTF32): the score tiles X = Q K^T and
    Y = dO V^T at or below the diagonal, P and dS from them (dS into the
    caller's B*H*T*T scratch, the reference's size), then dQ = dS K,
    dV = P^T dO and dK = dS^T Q as GEMMs over their causal ranges.  Ragged row
    tiles included; compared with the oracle and with the explicit-shape
    backward (CUDA-core kernels)."""
    import torch
    A.check(A.lib.attn_set_macro_shape(B, H, T, d))
    try:
        q, k, v = qkv(7 * T + d, B, T, H, d)
        do = synth.normal(8 * T + d, q.shape)
        ref, probs, _ = O.attn_forward(q, k, v, B, T, H, d, want_probs=True)
        rq, rk, rv = O.attn_backward(do, q, k, v, probs, B, T, H, d)
        qd, kd, vd, gd = dev(q), dev(k), dev(v), dev(do)
        att = torch.empty_like(qd)
        probs_buf = torch.empty(B * H * T * T, device="cuda")
        scratch = torch.full((B * H * T * T,), float("nan"), device="cuda")
        dq, dk, dv = (torch.full_like(qd, 7.0) for _ in range(3))
        torch.cuda.synchronize()
        A.lib.attn_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), att.data_ptr(), probs_buf.data_ptr())
        A.lib.attn_bwd(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), scratch.data_ptr(), gd.data_ptr(),
                       qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), probs_buf.data_ptr())
        torch.cuda.synchronize()
        assert rel_err(host(dq), rq) < F32_TOL
        assert rel_err(host(dk), rk) < F32_TOL
        assert rel_err(host(dv), rv) < F32_TOL
        o, lse = A.forward_t(qd, kd, vd, H, B)
        fq, fk, fv = A.backward_t(gd, qd, kd, vd, o, lse, H, B)
        torch.cuda.synchronize()
        assert rel_err(host(dq), host(fq)) < F32_TOL
        assert rel_err(host(dk), host(fk)) < F32_TOL
        assert rel_err(host(dv), host(fv)) < F32_TOL
        code = ctypes.c_int()
        A.check(A.lib.attn_device_error(0, ctypes.byref(code)))
        assert code.value == 0
    finally:
        A.lib.attn_set_macro_shape(4, 12, 1024, 128)


@pytest.mark.parametrize("B,H,T,d", [(2, 2, 260, 128), (1, 3, 128, 96)])
def test_backward_ex_tensor_core_workspace(A, B, H, T, d):
    """attn_bwd_ex at d 96 / 128 with a workspace of attn_bwd_tc_workspace_bytes:
    the tensor-core GEMMs over score tiles, against the oracle and against the
    CUDA-core kernels that the minimum workspace selects; accumulate = 1 keeps
    the CUDA-core kernels (the GEMMs set their outputs)."""
    import torch
    q, k, v = qkv(13 * T + d, B, T, H, d)
    do = synth.normal(14 * T + d, q.shape)
    _, probs, _ = O.attn_forward(q, k, v, B, T, H, d, want_probs=True)
    rq, rk, rv = O.attn_backward(do, q, k, v, probs, B, T, H, d)
    qd, kd, vd, gd = dev(q), dev(k), dev(v), dev(do)
    o, lse = A.forward_t(qd, kd, vd, H, B)
    shape = A.Shape(B, H, T, d, 0, 0)
    big = A.lib.attn_bwd_tc_workspace_bytes(ctypes.byref(shape))
    small = A.bwd_workspace_bytes(shape, A.F32)
    assert big > small
    outs = {}
    for name, nbytes in (("tc", big), ("ffma", small)):
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        r = [torch.full_like(qd, 7.0) for _ in range(3)]
        A.bwd_ex(shape, A.F32, gd.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(),
                 lse.data_ptr(), r[0].data_ptr(), r[1].data_ptr(), r[2].data_ptr(), 0, ws.data_ptr(), nbytes, 0)
        torch.cuda.synchronize()
        outs[name] = [host(t) for t in r]
        for got, want in zip(outs[name], (rq, rk, rv)):
            assert rel_err(got, want) < F32_TOL, name
    for a, b in zip(outs["tc"], outs["ffma"]):
        assert rel_err(a, b) < F32_TOL
    # accumulate = 1 with the large workspace adds, like train.c:372
    ws = torch.empty(big, dtype=torch.uint8, device="cuda")
    acc = [torch.ones_like(qd) for _ in range(3)]
    A.bwd_ex(shape, A.F32, gd.data_ptr(), qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(), lse.data_ptr(),
             acc[0].data_ptr(), acc[1].data_ptr(), acc[2].data_ptr(), 1, ws.data_ptr(), big, 0)
    torch.cuda.synchronize()
    for got, want in zip(acc, (rq, rk, rv)):
        assert rel_err(host(got) - 1.0, want) < F32_TOL


@pytest.mark.parametrize("B,H,T,d", [(1, 2, 1536, 128), (2, 3, 100, 128), (1, 2, 40, 64)])
def test_drop_in_lse_only_probs(A, B, H, T, d):
    """ATTN_PROBS_LSE: `probs` shrinks to B*H*T floats and `scratch` to the
    backward's workspace (the trainer-side edit that drops train_kaggle.cu's
    B*H*T*T a_probs and s_Dbuf), T < d+1 included; nothing past those sizes is
    written, and the backward reads the output from `att`."""
    import torch
    A.check(A.lib.attn_set_probs_mode(A.PROBS_LSE))
    try:
        A.check(A.lib.attn_set_macro_shape(B, H, T, d))
        q, k, v = qkv(23, B, T, H, d)
        do = synth.normal(24, q.shape)
        ref, probs, _ = O.attn_forward(q, k, v, B, T, H, d, want_probs=True)
        rq, rk, rv = O.attn_backward(do, q, k, v, probs, B, T, H, d)
        qd, kd, vd, gd = dev(q), dev(k), dev(v), dev(do)
        att = torch.empty_like(qd)
        n_lse = B * H * T
        n_ws = A.bwd_workspace_bytes(A.Shape(B, H, T, d, 0, 0), A.F32) // 4
        canary = 1234.5
        probs_buf = torch.full((n_lse + 4096,), canary, device="cuda")
        scratch = torch.full((n_ws + 4096,), canary, device="cuda")
        dq, dk, dv = (torch.full_like(qd, 7.0) for _ in range(3))
        torch.cuda.synchronize()
        A.lib.attn_fwd(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), att.data_ptr(), probs_buf.data_ptr())
        A.lib.attn_bwd(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), scratch.data_ptr(), gd.data_ptr(),
                       qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), probs_buf.data_ptr())
        torch.cuda.synchronize()
        assert rel_err(host(att), ref) < F32_TOL
        assert rel_err(host(dq), rq) < F32_TOL
        assert rel_err(host(dk), rk) < F32_TOL
        assert rel_err(host(dv), rv) < F32_TOL
        assert bool((probs_buf[n_lse:] == canary).all())
        assert bool((scratch[n_ws:] == canary).all())
    finally:
        A.lib.attn_set_probs_mode(A.PROBS_LSE_OUT)
        A.lib.attn_set_macro_shape(4, 12, 1024, 128)


# ---------------------------------------------------------------------------
# decode
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", ["decode_h4_d32", "decode_h2_d64"])
def test_cached_attention_golden(A, name):
    import torch
    z = golden(name)
    H, d, _ = (int(x) for x in z["shape"])
    kc, vc = dev(z["kcache"]), dev(z["vcache"])
    for i, pos in enumerate(z["positions"]):
        q = dev(z["q"][i])
        out = torch.empty_like(q)
        A.check(A.lib.attn_cached_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), int(pos),
                                            H, d, H * d, None))
        torch.cuda.synchronize()
        assert rel_err(host(out), z["out"][i]) < F32_TOL


# (24, 32, ...) and d 96 take the split kernels, the others the single-pass
# kernel for small calls; (16, 64, 8, 3000) splits one sequence over ~40 CTAs.
@pytest.mark.parametrize("H,d,n_seq,max_len", [(16, 64, 8, 3000), (16, 32, 5, 700), (4, 128, 3, 1500),
                                               (2, 96, 4, 257), (16, 64, 2, 1), (24, 32, 3, 500),
                                               (8, 128, 1, 5000), (1, 32, 200, 37)])
def test_ragged_decode_f32_vs_oracle(A, H, d, n_seq, max_len):
    import torch
    lens = synth.uniform_int(H * d + n_seq, n_seq, 1, max_len)
    lens[0] = max_len
    cap = max_len
    kc = synth.normal(31, (n_seq * cap, H * d))
    vc = synth.normal(32, (n_seq * cap, H * d))
    q = synth.normal(33, (n_seq, H * d))
    out = A.decode_t(dev(q), dev(kc), dev(vc), dev(lens), H, cap, max_len)
    torch.cuda.synchronize()
    for s in range(n_seq):
        ref = O.cached_attention(q[s], kc[s * cap:(s + 1) * cap], vc[s * cap:(s + 1) * cap], int(lens[s]) - 1, H, d)
        assert rel_err(host(out)[s], ref) < F32_TOL, s


def test_decode_pointer_array_layers(A):
    """attn_decode_ptrs_ex over per-layer slabs (KVCache.k[l], model.h:43)."""
    import torch
    L, H, d, cap, pos = 4, 16, 32, 640, 600
    ks = [synth.normal(40 + l, (cap, H * d)) for l in range(L)]
    vs = [synth.normal(50 + l, (cap, H * d)) for l in range(L)]
    q = synth.normal(60, (L, H * d))
    kd = [dev(x) for x in ks]
    vd = [dev(x) for x in vs]
    kp = torch.tensor([t.data_ptr() for t in kd], dtype=torch.int64, device="cuda")
    vp = torch.tensor([t.data_ptr() for t in vd], dtype=torch.int64, device="cuda")
    lens = torch.full((L,), pos + 1, dtype=torch.int32, device="cuda")
    qd = dev(q)
    out = torch.empty_like(qd)
    shape = A.DecodeShape(L, H, d, A.F32, 0, cap, cap)
    A.check(A.lib.attn_decode_ptrs_ex(ctypes.byref(shape), qd.data_ptr(), kp.data_ptr(), vp.data_ptr(), None, None,
                                      lens.data_ptr(), out.data_ptr(), None, 0, None))
    torch.cuda.synchronize()
    for l in range(L):
        ref = O.ref_cached_attention(q[l], ks[l], vs[l], pos, H, d, 1024) if O.ref_available() else \
            O.cached_attention(q[l], ks[l], vs[l], pos, H, d)
        assert rel_err(host(out)[l], ref) < F32_TOL


def test_quantiser_bit_exact(A):
    import torch
    z = golden("quant_h4_d32")
    H, d = (int(x) for x in z["shape"])
    codes, scales = A.quantize_int8_t(dev(z["x"]), H)
    torch.cuda.synchronize()
    assert np.array_equal(host(codes), z["codes"])
    assert np.array_equal(host(scales).view(np.uint32), z["scales"].view(np.uint32))
    x = synth.normal(5, (333, 16 * 64), 0, 3.0)
    c2, s2 = A.quantize_int8_t(dev(x), 16)
    rc, rs = O.quantize_kv_int8(x, 16, 64)
    assert np.array_equal(host(c2), rc) and np.array_equal(host(s2).view(np.uint32), rs.view(np.uint32))


def test_int8_decode_golden(A):
    import torch
    z = golden("int8_decode_h2_d64")
    H, d, _ = (int(x) for x in z["shape"])
    pos = int(z["pos"])
    lens = torch.tensor([pos + 1], dtype=torch.int32, device="cuda")
    out = A.decode_t(dev(z["q"][None, :]), dev(z["kcodes"]), dev(z["vcodes"]), lens, H, pos + 1, pos + 1,
                     kscale=dev(z["kscale"]), vscale=dev(z["vscale"]))
    torch.cuda.synchronize()
    assert rel_err(host(out)[0], z["out"]) < F32_TOL


@pytest.mark.parametrize("H,d,n_seq,max_len", [(16, 64, 6, 4000), (16, 32, 3, 900), (2, 128, 3, 333)])
def test_ragged_decode_int8_vs_dequantised_oracle(A, H, d, n_seq, max_len):
    import torch
    lens = synth.uniform_int(3 * H + d, n_seq, 1, max_len)
    cap = max_len
    kc = synth.normal(71, (n_seq * cap, H * d))
    vc = synth.normal(72, (n_seq * cap, H * d))
    q = synth.normal(73, (n_seq, H * d))
    kq, ksc = A.quantize_int8_t(dev(kc), H)
    vq, vsc = A.quantize_int8_t(dev(vc), H)
    out = A.decode_t(dev(q), kq, vq, dev(lens), H, cap, max_len, kscale=ksc, vscale=vsc)
    torch.cuda.synchronize()
    kd = O.dequantize_kv_int8(host(kq), host(ksc), H, d)
    vd = O.dequantize_kv_int8(host(vq), host(vsc), H, d)
    for s in range(n_seq):
        ref = O.cached_attention(q[s], kd[s * cap:(s + 1) * cap], vd[s * cap:(s + 1) * cap], int(lens[s]) - 1, H, d)
        assert rel_err(host(out)[s], ref) < F32_TOL
        # informational bound against the un-quantised cache
        ref32 = O.cached_attention(q[s], kc[s * cap:(s + 1) * cap], vc[s * cap:(s + 1) * cap], int(lens[s]) - 1, H, d)
        assert rel_err(host(out)[s], ref32) < 5e-2


def test_decode_caller_workspace_and_reuse(A):
    import torch
    H, d, n_seq, max_len = 16, 64, 4, 2048
    lens = synth.uniform_int(9, n_seq, 1000, max_len)
    kc = synth.normal(81, (n_seq * max_len, H * d))
    vc = synth.normal(82, (n_seq * max_len, H * d))
    q = synth.normal(83, (n_seq, H * d))
    shape = A.DecodeShape(n_seq, H, d, A.F32, 0, max_len, max_len)
    ws = torch.zeros(A.decode_workspace_bytes(shape), dtype=torch.uint8, device="cuda")
    outs = [host(A.decode_t(dev(q), dev(kc), dev(vc), dev(lens), H, max_len, max_len, workspace=ws))
            for _ in range(3)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])
    ref = O.cached_attention(q[1], kc[max_len:2 * max_len], vc[max_len:2 * max_len], int(lens[1]) - 1, H, d)
    assert rel_err(outs[0][1], ref) < F32_TOL


def test_decode_padded_rows_and_dirty_workspace(A):
    """Cache rows padded past H*d (row copies one by one) and a caller workspace
    full of stale bytes: the merge tickets carry the call's generation, so old
    contents never count."""
    import torch
    H, d, n_seq, max_len, pad = 16, 32, 3, 900, 16
    lens = synth.uniform_int(77, n_seq, 1, max_len)
    lens[1] = max_len
    kc = synth.normal(91, (n_seq * max_len, H * d + pad))
    vc = synth.normal(92, (n_seq * max_len, H * d + pad))
    q = synth.normal(93, (n_seq, H * d))
    kd, vd = dev(kc)[:, :H * d], dev(vc)[:, :H * d]
    shape = A.DecodeShape(n_seq, H, d, A.F32, H * d + pad, max_len, max_len)
    ws = torch.full((A.decode_workspace_bytes(shape),), 0xFF, dtype=torch.uint8, device="cuda")
    for _ in range(2):
        out = A.decode_t(dev(q), kd, vd, dev(lens), H, max_len, max_len, workspace=ws)
        torch.cuda.synchronize()
        for s_ in range(n_seq):
            ref = O.cached_attention(q[s_], kc[s_ * max_len:(s_ + 1) * max_len, :H * d],
                                     vc[s_ * max_len:(s_ + 1) * max_len, :H * d], int(lens[s_]) - 1, H, d)
            assert rel_err(host(out)[s_], ref) < F32_TOL, s_
        ws.random_(0, 256)


def test_decode_bounded_wait_timeout_path(A):
    """Failure detection without a fault: a test hook makes one warp of the
    TMA-ring decode kernel wait on a barrier nothing arrives at.  The
    bounded wait runs out, the kernel records its code in the device error
    word, lets its in-flight copies land and returns; the next call is
    correct and leaves the error word clear."""
    import torch
    H, d, n_seq, max_len = 16, 32, 40, 640         # 640 (sequence, head) units: the ring kernel's calls
    lens = np.full(n_seq, max_len, np.int32)
    kc = synth.normal(94, (n_seq * max_len, H * d))
    vc = synth.normal(95, (n_seq * max_len, H * d))
    q = synth.normal(96, (n_seq, H * d))
    qd, kd, vd, ld = dev(q), dev(kc), dev(vc), dev(lens)
    code = ctypes.c_int()
    A.check(A.lib.attn_device_error(0, ctypes.byref(code)))       # clear
    A.check(A.lib.attn_debug_decode_timeout(1, 200000))
    try:
        A.decode_t(qd, kd, vd, ld, H, max_len, max_len)
        torch.cuda.synchronize()
    finally:
        A.check(A.lib.attn_debug_decode_timeout(0, 0))             # disarmed whatever ran
    A.check(A.lib.attn_device_error(0, ctypes.byref(code)))
    assert code.value == 0x32f
    out = A.decode_t(qd, kd, vd, ld, H, max_len, max_len)
    torch.cuda.synchronize()
    A.check(A.lib.attn_device_error(0, ctypes.byref(code)))
    assert code.value == 0
    for s_ in (0, 17, 39):
        ref = O.cached_attention(q[s_], kc[s_ * max_len:(s_ + 1) * max_len], vc[s_ * max_len:(s_ + 1) * max_len],
                                 max_len - 1, H, d)
        assert rel_err(host(out)[s_], ref) < F32_TOL


def test_decode_bad_length_sets_device_error_word(A):
    """Failure detection without a fault: an out-of-range length is clamped,
    recorded in the device error word, and the context stays usable."""
    import torch
    H, d, cap = 2, 64, 100
    kc, vc = dev(synth.normal(1, (cap, H * d))), dev(synth.normal(2, (cap, H * d)))
    q = dev(synth.normal(3, (1, H * d)))
    code = ctypes.c_int()
    A.check(A.lib.attn_device_error(0, ctypes.byref(code)))       # clear
    out = A.decode_t(q, kc, vc, dev(np.array([cap + 50], np.int32)), H, cap, cap)
    torch.cuda.synchronize()
    A.check(A.lib.attn_device_error(0, ctypes.byref(code)))
    assert code.value != 0
    assert np.isfinite(host(out)).all()
    A.check(A.lib.attn_device_error(0, ctypes.byref(code)))
    assert code.value == 0


def test_kv_cache_alloc_append_decode(A):
    import torch
    for kv in (A.F32, A.I8):
        c = A.KVCache()
        L, cap, H, d = 3, 64, 4, 32
        A.check(A.lib.attn_kv_cache_alloc(ctypes.byref(c), L, cap, H, d, kv))
        try:
            rows_k = synth.normal(10 + kv, (cap, H * d))
            rows_v = synth.normal(20 + kv, (cap, H * d))
            kd, vd = dev(rows_k), dev(rows_v)
            for pos in range(40):
                A.check(A.lib.attn_kv_cache_append(ctypes.byref(c), 1, pos, kd[pos].data_ptr(), vd[pos].data_ptr(),
                                                   None))
            q = dev(synth.normal(30, (1, H * d)))
            out = torch.empty_like(q)
            lens = torch.tensor([40], dtype=torch.int32, device="cuda")
            shape = A.DecodeShape(1, H, d, kv, 0, cap, cap)
            A.check(A.lib.attn_decode_ex(ctypes.byref(shape), q.data_ptr(), c.k[1], c.v[1], c.kscale[1], c.vscale[1],
                                         lens.data_ptr(), out.data_ptr(), None, 0, None))
            torch.cuda.synchronize()
            kr, vr = rows_k[:40], rows_v[:40]
            if kv == A.I8:
                kr = O.dequantize_kv_int8(*O.quantize_kv_int8(kr, H, d), H, d)
                vr = O.dequantize_kv_int8(*O.quantize_kv_int8(vr, H, d), H, d)
            ref = O.cached_attention(host(q)[0], kr, vr, 39, H, d)
            assert rel_err(host(out)[0], ref) < F32_TOL
        finally:
            A.check(A.lib.attn_kv_cache_free(ctypes.byref(c)))


def test_gather_permute(A):
    import torch
    G, B, T, H, d = 4, 2, 33, 8, 32
    staging = synth.normal(5, (G, B, T, H // G, d))
    out = A.gather_permute_t(dev(staging).reshape(-1, d), G, B, T, H, d)
    torch.cuda.synchronize()
    ref = staging.transpose(1, 2, 0, 3, 4).reshape(B * T, H * d)
    assert np.array_equal(host(out), ref)


# ---------------------------------------------------------------------------
# INT8 streaming decode kernel (1024-code rows): the paths its producer takes
# ---------------------------------------------------------------------------
def _int8_decode_case(A, H, d, lens, cap, row_pad=0, seed=90, mutate=None):
    """Quantised caches (optionally with padded rows), decode, and the oracle
    over the dequantised cache; returns (out, refs).  `mutate(q, kscale,
    vscale)` may edit the query (numpy) and the scales (device) in place first."""
    import torch
    n_seq = len(lens)
    width = H * d
    kc = synth.normal(seed, (n_seq * cap, width))
    vc = synth.normal(seed + 1, (n_seq * cap, width))
    q = synth.normal(seed + 2, (n_seq, width))
    kq, ksc = A.quantize_int8_t(dev(kc), H)
    vq, vsc = A.quantize_int8_t(dev(vc), H)
    if mutate:
        mutate(q, ksc, vsc)
    if row_pad:
        # the same codes in rows of width + row_pad bytes (strided slabs)
        kp = torch.zeros((n_seq * cap, width + row_pad), dtype=torch.int8, device="cuda")
        vp = torch.zeros_like(kp)
        kp[:, :width] = kq
        vp[:, :width] = vq
        kq_in, vq_in = kp[:, :width], vp[:, :width]
    else:
        kq_in, vq_in = kq, vq
    lens_t = dev(np.asarray(lens, dtype=np.int32))
    out = A.decode_t(dev(q), kq_in, vq_in, lens_t, H, cap, cap, kscale=ksc, vscale=vsc)
    torch.cuda.synchronize()
    kd = O.dequantize_kv_int8(host(kq), host(ksc), H, d)
    vd = O.dequantize_kv_int8(host(vq), host(vsc), H, d)
    refs = [O.cached_attention(q[s], kd[s * cap:(s + 1) * cap], vd[s * cap:(s + 1) * cap], int(lens[s]) - 1, H, d)
            for s in range(n_seq)]
    return host(out), refs


@pytest.mark.parametrize("H,d", [(16, 64), (8, 128)])
def test_int8_stream_piece_boundaries(A, H, d):
    """Lengths of 1 row, exactly one piece, one piece + 1, several pieces and the
    capacity: every branch of the piece table and of the last, partial block."""
    cap = 2100
    lens = [1, 2, 15, 16, 17, 64, 65, 511, 512, 513, 1024, 1500, 2099, cap]
    out, refs = _int8_decode_case(A, H, d, lens, cap)
    for s, ref in enumerate(refs):
        assert rel_err(out[s], ref) < F32_TOL, (s, lens[s])


@pytest.mark.parametrize("H,d", [(16, 64), (8, 128)])
def test_int8_decode_signed_scales_and_zero_query(A, H, d):
    """Scales of either sign (the dequantised value is code * scale whatever
    its sign), a zero query row and a zero value scale, at lengths on and
    around the 128-row tile and the 512-row piece."""
    lens = [1, 127, 128, 129, 383, 384, 385, 511, 512, 513, 1030]
    cap = 1040

    def mutate(q, ksc, vsc):
        ksc[::3] *= -1
        vsc[::5] *= -1
        vsc[7] = 0.0
        q[3] = 0.0

    out, refs = _int8_decode_case(A, H, d, lens, cap, seed=150, mutate=mutate)
    for s, ref in enumerate(refs):
        assert rel_err(out[s], ref) < F32_TOL, (s, lens[s])


@pytest.mark.parametrize("H,d", [(16, 64), (8, 128)])
def test_int8_decode_fewer_rows_than_sms(A, H, d):
    """Fewer cache rows in all than SMs: most CTAs get an empty share, and a
    sequence's rows are spread over several CTAs with empty ones between."""
    lens = [1, 3, 2, 7, 1]
    out, refs = _int8_decode_case(A, H, d, lens, 8, seed=160)
    for s, ref in enumerate(refs):
        assert rel_err(out[s], ref) < F32_TOL, (s, lens[s])


def test_int8_stream_strided_rows(A):
    """Rows wider than H*d (per-row bulk copies instead of one copy per block)."""
    lens = [300, 1, 777]
    out, refs = _int8_decode_case(A, 16, 64, lens, 800, row_pad=64, seed=95)
    for s, ref in enumerate(refs):
        assert rel_err(out[s], ref) < F32_TOL, s


def test_int8_stream_pointer_slabs(A):
    """attn_decode_ptrs_ex with INT8 slabs and per-slab scale arrays."""
    import torch
    L, H, d, cap = 3, 16, 64, 700
    lens = np.asarray([700, 123, 512], dtype=np.int32)
    ks = [synth.normal(110 + l, (cap, H * d)) for l in range(L)]
    vs = [synth.normal(120 + l, (cap, H * d)) for l in range(L)]
    q = synth.normal(130, (L, H * d))
    kq, ksc, vq, vsc = [], [], [], []
    for l in range(L):
        a, b = A.quantize_int8_t(dev(ks[l]), H)
        c, e = A.quantize_int8_t(dev(vs[l]), H)
        kq.append(a), ksc.append(b), vq.append(c), vsc.append(e)
    ptrs = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")
    kp, vp, ksp, vsp = ptrs(kq), ptrs(vq), ptrs(ksc), ptrs(vsc)
    qd = dev(q)
    out = torch.empty_like(qd)
    lens_t = dev(lens)
    shape = A.DecodeShape(L, H, d, A.I8, 0, cap, cap)
    A.check(A.lib.attn_decode_ptrs_ex(ctypes.byref(shape), qd.data_ptr(), kp.data_ptr(), vp.data_ptr(),
                                      ksp.data_ptr(), vsp.data_ptr(), lens_t.data_ptr(), out.data_ptr(), None, 0,
                                      None))
    torch.cuda.synchronize()
    for l in range(L):
        kd = O.dequantize_kv_int8(host(kq[l]), host(ksc[l]), H, d)
        vd = O.dequantize_kv_int8(host(vq[l]), host(vsc[l]), H, d)
        ref = O.cached_attention(q[l], kd, vd, int(lens[l]) - 1, H, d)
        assert rel_err(host(out)[l], ref) < F32_TOL, l


def test_int8_decode_many_sequences_fallback(A):
    """More sequences than the stream kernel's piece table holds (1024): the
    split kernels take the call, with the same results."""
    n_seq, H, d, cap = 1030, 16, 64, 24
    lens = synth.uniform_int(140, n_seq, 1, cap)
    out, refs = _int8_decode_case(A, H, d, [int(x) for x in lens], cap, seed=140)
    for s in range(0, n_seq, 97):
        assert rel_err(out[s], refs[s]) < F32_TOL, s
