"""The CPU restatement (oracle/attn_oracle.c) pinned against fixtures the
reference's own code produced (tests/golden/make_golden.py)."""
import numpy as np
import pytest

from conftest import golden, rel_err
from oracle import oracle as O

F32_TOL = 1e-5


@pytest.mark.parametrize("name", ["fwd_h4_d32", "fwd_h2_d64", "fwd_h2_d128", "fwd_h2_d96", "fwd_t1"])
def test_forward_matches_reference(name):
    z = golden(name)
    B, T, H, d = (int(x) for x in z["shape"])
    att, probs, lse = O.attn_forward(z["q"], z["k"], z["v"], B, T, H, d, want_probs=True)
    assert rel_err(att, z["att"]) < F32_TOL
    assert rel_err(probs, z["probs"]) < F32_TOL
    # lse is the statistic the GPU path keeps instead of probs
    assert rel_err(O.lse_to_probs(z["q"], z["k"], lse, B, T, H, d), z["probs"]) < F32_TOL


@pytest.mark.parametrize("name", ["fwd_h4_d32", "fwd_h2_d64"])
def test_forward_f64_twin(name):
    z = golden(name)
    B, T, H, d = (int(x) for x in z["shape"])
    assert rel_err(O.attn_forward_f64(z["q"], z["k"], z["v"], B, T, H, d), z["att"]) < F32_TOL


@pytest.mark.parametrize("name", ["bwd_h2_d64", "bwd_h4_d32"])
def test_backward_matches_reference(name):
    z = golden(name)
    B, T, H, d = (int(x) for x in z["shape"])
    _, probs, _ = O.attn_forward(z["q"], z["k"], z["v"], B, T, H, d, want_probs=True)
    dq, dk, dv = O.attn_backward(z["do"], z["q"], z["k"], z["v"], probs, B, T, H, d)
    assert rel_err(dq, z["dq"]) < F32_TOL
    assert rel_err(dk, z["dk"]) < F32_TOL
    assert rel_err(dv, z["dv"]) < F32_TOL


def test_backward_accumulates_like_train_c():
    z = golden("bwd_h4_d32")
    B, T, H, d = (int(x) for x in z["shape"])
    _, probs, _ = O.attn_forward(z["q"], z["k"], z["v"], B, T, H, d, want_probs=True)
    dq, dk, dv = O.attn_backward(z["do"], z["q"], z["k"], z["v"], probs, B, T, H, d)
    dq2, dk2, dv2 = O.attn_backward(2 * z["do"], z["q"], z["k"], z["v"], probs, B, T, H, d)
    # linear in dO: the zero-started accumulation of 2*dO is twice dO's
    assert rel_err(dq2, 2 * dq) < F32_TOL and rel_err(dv2, 2 * dv) < F32_TOL


@pytest.mark.parametrize("name", ["decode_h4_d32", "decode_h2_d64"])
def test_decode_matches_reference(name):
    z = golden(name)
    H, d, _ = (int(x) for x in z["shape"])
    for i, pos in enumerate(z["positions"]):
        out = O.cached_attention(z["q"][i], z["kcache"], z["vcache"], int(pos), H, d)
        assert rel_err(out, z["out"][i]) < F32_TOL
        out64 = O.cached_attention(z["q"][i], z["kcache"], z["vcache"], int(pos), H, d, f64=True)
        assert rel_err(out64, z["out"][i]) < F32_TOL


def test_quantiser_bit_exact_vs_reference():
    z = golden("quant_h4_d32")
    H, d = (int(x) for x in z["shape"])
    codes, scales = O.quantize_kv_int8(z["x"], H, d)
    assert np.array_equal(codes, z["codes"])
    assert np.array_equal(scales.view(np.uint32), z["scales"].view(np.uint32))
    # the fixture pins the edge cases: ties round half away from zero
    assert list(z["codes"][1, :9]) == [127, 3, -3, 1, -1, 2, -2, 127, -127]
    assert np.float32(z["scales"][0, 0]) == np.float32(1e-8) / np.float32(127.0)


def test_int8_decode_matches_reference():
    z = golden("int8_decode_h2_d64")
    H, d, _ = (int(x) for x in z["shape"])
    kd = O.dequantize_kv_int8(z["kcodes"], z["kscale"], H, d)
    vd = O.dequantize_kv_int8(z["vcodes"], z["vscale"], H, d)
    out = O.cached_attention(z["q"], kd, vd, int(z["pos"]), H, d)
    assert rel_err(out, z["out"]) < F32_TOL


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")
def test_restatement_vs_live_reference_random_shapes():
    import synth
    for seed, (B, T, H, d) in enumerate([(1, 130, 2, 64), (3, 5, 4, 32), (1, 64, 1, 64)]):
        q = synth.normal(900 + seed, (B * T, H * d), 0, 0.5)
        k = synth.normal(910 + seed, (B * T, H * d), 0, 0.5)
        v = synth.normal(920 + seed, (B * T, H * d), 0, 0.5)
        att, probs, _ = O.attn_forward(q, k, v, B, T, H, d, want_probs=True)
        ra, rp = O.ref_attention_forward(q, k, v, B, T, H, d)
        assert rel_err(att, ra) < F32_TOL and rel_err(probs, rp) < F32_TOL


@pytest.mark.parametrize("name", ["qkv_m72_k96_n64", "qkv_m37_k52_n36"])
def test_qkv_projection_matches_reference(name):
    """matmul_forward restated (train.c:181-211) against the reference's own
    object, for the three projections of train.c:517-519; both of the
    reference's code paths (micro-kernel and i-k-j loop) are covered."""
    z = golden(name)
    ws, bs = (z["wq"], z["wk"], z["wv"]), (z["bq"], z["bk"], z["bv"])
    for out, want in zip(O.qkv_proj(z["x"], ws, bs), (z["q"], z["k"], z["v"])):
        assert rel_err(out, want) < F32_TOL
    for out, want in zip(O.qkv_proj(z["x"], ws, bs, f64=True), (z["q"], z["k"], z["v"])):
        assert rel_err(out, want) < F32_TOL


def test_matmul_restatement_vs_live_reference():
    import synth
    for seed, (M, K, N) in enumerate([(64, 128, 96), (9, 20, 12), (128, 1536, 16)]):
        x = synth.normal(950 + seed, (M, K))
        w = synth.normal(960 + seed, (K, N), 0, 0.02)
        b = synth.normal(970 + seed, (N,), 0, 0.1)
        assert rel_err(O.matmul_forward(x, w, b), O.ref_matmul_forward(x, w, b)) < F32_TOL
        assert rel_err(O.matmul_forward(x, w, None), O.ref_matmul_forward(x, w, None)) < F32_TOL
