"""The five workloads of the benchmark at their full sizes.  The oracle checks
sampled (batch, head) units / sequences / decode steps exactly; whole-tensor
properties cover the rest: V = 1 gives O = 1 (softmax rows sum to one),
linearity in V, and finiteness."""
import numpy as np
import pytest

from conftest import rel_err
from oracle import oracle as O

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
BF16_FWD_TOL = 2e-2
BF16_BWD_TOL = 3e-2


@pytest.fixture(scope="module")
def A(cuda):
    import attn_b200
    return attn_b200


def unit(x, b, h, T, d):
    """(B*T, H*d) tensor -> the (T, d) slice of batch b, head h, as numpy fp32."""
    return x[b * T:(b + 1) * T, h * d:(h + 1) * d].float().cpu().numpy()


def slab(x, b, h0, nh, T, d):
    """(B*T, H*d) tensor -> the (T, nh*d) columns of heads h0..h0+nh-1 of batch b."""
    return np.ascontiguousarray(x[b * T:(b + 1) * T, h0 * d:(h0 + nh) * d].float().cpu().numpy())


def gen(shape, seed, std, dtype):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(shape, generator=g, device="cuda") * std).to(dtype)


@pytest.mark.parametrize("cfg", ["c2_f32", "c3_f32", "c3_bf16"])
def test_prefill_full_size(A, cfg):
    import torch
    B, H, T = 8, 16, 1024
    d = 32 if cfg.startswith("c2") else 64
    dt = torch.bfloat16 if cfg.endswith("bf16") else torch.float32
    q, k, v = (gen((B * T, H * d), s, 0.5, dt) for s in (1, 2, 3))
    o, lse = A.forward_t(q, k, v, H, B)
    torch.cuda.synchronize()
    assert torch.isfinite(o.float()).all()
    tol = BF16_FWD_TOL if dt == torch.bfloat16 else F32_TOL
    for b, h in [(0, 0), (7, 15), (3, 9)]:
        ref, _, _ = O.attn_forward(unit(q, b, h, T, d), unit(k, b, h, T, d), unit(v, b, h, T, d), 1, T, 1, d)
        assert rel_err(unit(o, b, h, T, d), ref) < tol
    # V = 1  =>  O = 1 for every row of every head
    ones = torch.ones_like(v)
    o1, _ = A.forward_t(q, k, ones, H, B)
    torch.cuda.synchronize()
    assert (o1.float() - 1).abs().max().item() < (1e-2 if dt == torch.bfloat16 else 1e-5)
    # linearity in V
    v2 = gen((B * T, H * d), 4, 0.5, dt)
    o2, _ = A.forward_t(q, k, v2, H, B)
    o12, _ = A.forward_t(q, k, (v.float() + v2.float()).to(dt), H, B)
    torch.cuda.synchronize()
    diff = (o12.float() - o.float() - o2.float()).abs().max().item()
    assert diff < (5e-2 if dt == torch.bfloat16 else 1e-5)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_backward_full_size_c5(A, dtype):
    import torch
    B, H, T, d = 4, 16, 4096, 64
    dt = torch.bfloat16 if dtype == "bf16" else torch.float32
    q, k, v = (gen((B * T, H * d), s, 0.5, dt) for s in (11, 12, 13))
    do = gen((B * T, H * d), 14, 1.0, dt)
    o, lse = A.forward_t(q, k, v, H, B)
    dq, dk, dv = A.backward_t(do, q, k, v, o, lse, H, B)
    torch.cuda.synchronize()
    for t in (dq, dk, dv):
        assert torch.isfinite(t.float()).all()
    tol = BF16_BWD_TOL if dt == torch.bfloat16 else F32_TOL
    # Sixteen (batch, head) units -- every head of batch 2 -- against the
    # reference's own train.c backward (OpenMP over the heads), or eight of
    # them against the restatement where the reference objects are absent.
    use_ref = O.ref_available()
    for b, h0, nh in ((2, 0, 16),) if use_ref else ((2, 4, 8),):
        qu, ku, vu, gu = (slab(x, b, h0, nh, T, d) for x in (q, k, v, do))
        if use_ref:
            _, probs = O.ref_attention_forward(qu, ku, vu, 1, T, nh, d)
            rq, rk, rv = O.ref_attention_backward(gu, qu, ku, vu, probs, 1, T, nh, d)
        else:
            _, probs, _ = O.attn_forward(qu, ku, vu, 1, T, nh, d, want_probs=True)
            rq, rk, rv = O.attn_backward(gu, qu, ku, vu, probs, 1, T, nh, d)
        for h in range(nh):
            cols = slice(h * d, (h + 1) * d)
            assert rel_err(unit(dq, b, h0 + h, T, d), rq[:, cols]) < tol, (b, h0 + h)
            assert rel_err(unit(dk, b, h0 + h, T, d), rk[:, cols]) < tol, (b, h0 + h)
            assert rel_err(unit(dv, b, h0 + h, T, d), rv[:, cols]) < tol, (b, h0 + h)


def test_drop_ins_at_trainer_shape(A):
    """attn_fwd / attn_bwd at the reference GPU trainer's own shape (B4 H12
    T1024 d128, gpu_kernels.h:17-31) with the trainer's buffer sizes, the
    backward's products all on the tensor cores: every head of batch 1 against
    the reference's own train.c attention (the restatement where the reference
    objects are absent)."""
    import ctypes
    import torch
    B, H, T, d = 4, 12, 1024, 128
    A.check(A.lib.attn_set_macro_shape(B, H, T, d))
    q, k, v = (gen((B * T, H * d), s, 0.5, torch.float32) for s in (21, 22, 23))
    do = gen((B * T, H * d), 24, 1.0, torch.float32)
    att = torch.empty_like(q)
    probs = torch.empty(B * H * T * T, device="cuda")
    scratch = torch.empty(B * H * T * T, device="cuda")
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    torch.cuda.synchronize()
    P = ctypes.c_void_p
    A.lib.attn_fwd(P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(att.data_ptr()), P(probs.data_ptr()))
    A.lib.attn_bwd(P(dq.data_ptr()), P(dk.data_ptr()), P(dv.data_ptr()), P(scratch.data_ptr()), P(do.data_ptr()),
                   P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(probs.data_ptr()))
    torch.cuda.synchronize()
    b = 1
    qu, ku, vu, gu = (slab(x, b, 0, H, T, d) for x in (q, k, v, do))
    if O.ref_available():
        ra, probs_r = O.ref_attention_forward(qu, ku, vu, 1, T, H, d)
        rq, rk, rv = O.ref_attention_backward(gu, qu, ku, vu, probs_r, 1, T, H, d)
    else:
        ra, probs_r, _ = O.attn_forward(qu, ku, vu, 1, T, H, d, want_probs=True)
        rq, rk, rv = O.attn_backward(gu, qu, ku, vu, probs_r, 1, T, H, d)
    for h in range(H):
        cols = slice(h * d, (h + 1) * d)
        assert rel_err(unit(att, b, h, T, d), ra[:, cols]) < F32_TOL, h
        assert rel_err(unit(dq, b, h, T, d), rq[:, cols]) < F32_TOL, h
        assert rel_err(unit(dk, b, h, T, d), rk[:, cols]) < F32_TOL, h
        assert rel_err(unit(dv, b, h, T, d), rv[:, cols]) < F32_TOL, h


def test_c1_layer_decode_full_run(A):
    """16 layers x 128 steps at d_model 512 = 16 x 32, caches of 512 prior rows."""
    import ctypes
    import torch
    L, H, d, prior, steps = 16, 16, 32, 512, 128
    cap = prior + steps
    kc = [gen((cap, H * d), 100 + l, 1.0, torch.float32) for l in range(L)]
    vc = [gen((cap, H * d), 200 + l, 1.0, torch.float32) for l in range(L)]
    q = gen((steps, L, H * d), 300, 1.0, torch.float32)
    kp = torch.tensor([t.data_ptr() for t in kc], dtype=torch.int64, device="cuda")
    vp = torch.tensor([t.data_ptr() for t in vc], dtype=torch.int64, device="cuda")
    out = torch.empty_like(q)
    shape = A.DecodeShape(L, H, d, A.F32, 0, cap, cap)
    for s in range(steps):
        lens = torch.full((L,), prior + s + 1, dtype=torch.int32, device="cuda")
        A.check(A.lib.attn_decode_ptrs_ex(ctypes.byref(shape), q[s].data_ptr(), kp.data_ptr(), vp.data_ptr(), None,
                                          None, lens.data_ptr(), out[s].data_ptr(), None, 0, None))
    torch.cuda.synchronize()
    for s, l in [(0, 0), (127, 15), (64, 7)]:
        ref = O.cached_attention(q[s, l].cpu().numpy(), kc[l].cpu().numpy(), vc[l].cpu().numpy(), prior + s, H, d)
        assert rel_err(out[s, l].cpu().numpy(), ref) < F32_TOL


@pytest.mark.parametrize("kv", ["f32", "int8"])
def test_c4_ragged_decode_full_size(A, kv):
    import synth
    import torch
    n_seq, H, d, max_len = 64, 16, 64, 8192
    lens_h = synth.uniform_int(2024, n_seq, 1, max_len)
    cap = int(lens_h.max())
    kc = gen((n_seq * cap, H * d), 41, 1.0, torch.float32)
    vc = gen((n_seq * cap, H * d), 42, 1.0, torch.float32)
    q = gen((n_seq, H * d), 43, 1.0, torch.float32)
    lens = torch.from_numpy(lens_h).cuda()
    if kv == "int8":
        kq, ks = A.quantize_int8_t(kc, H)
        vq, vs = A.quantize_int8_t(vc, H)
        out = A.decode_t(q, kq, vq, lens, H, cap, cap, kscale=ks, vscale=vs)
    else:
        out = A.decode_t(q, kc, vc, lens, H, cap, cap)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    for s in (0, 17, 63, int(np.argmax(lens_h)), int(np.argmin(lens_h))):
        rows = slice(s * cap, s * cap + int(lens_h[s]))
        if kv == "int8":
            kr = O.dequantize_kv_int8(kq[rows].cpu().numpy(), ks[rows].cpu().numpy(), H, d)
            vr = O.dequantize_kv_int8(vq[rows].cpu().numpy(), vs[rows].cpu().numpy(), H, d)
        else:
            kr, vr = kc[rows].cpu().numpy(), vc[rows].cpu().numpy()
        ref = O.cached_attention(q[s].cpu().numpy(), kr, vr, int(lens_h[s]) - 1, H, d)
        assert rel_err(out[s].cpu().numpy(), ref) < F32_TOL
