"""attn_decode_static_ex: the decode entry point for callers that cannot
allocate device memory (a generation loop whose memory belongs to another
allocator, or one that must not let cudaMalloc synchronise the device).  It
keeps its scratch in a fixed array inside the library instead of a caller or
library allocation.  Its results must equal the regular attn_decode_ex's, call
after call, since every call reuses the same array.

This file is named to be collected last, so that a run stopping at the first
failure has run every other test first; it also passes run alone."""
import ctypes

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5


def _case(A, kv, seed):
    import torch
    import synth
    H, d, n_seq, max_len = 16, 64, 8, 3000          # several splits per sequence
    lens = synth.uniform_int(seed, n_seq, 1, max_len)
    lens[0] = max_len
    kc = torch.from_numpy(synth.normal(seed + 1, (n_seq * max_len, H * d))).cuda()
    vc = torch.from_numpy(synth.normal(seed + 2, (n_seq * max_len, H * d))).cuda()
    q = torch.from_numpy(synth.normal(seed + 3, (n_seq, H * d))).cuda()
    ks = vs = None
    if kv == A.I8:
        kc, ks = A.quantize_int8_t(kc, H)
        vc, vs = A.quantize_int8_t(vc, H)
    shape = A.DecodeShape(n_seq, H, d, kv, 0, max_len, max_len)
    return shape, q, kc, vc, ks, vs, torch.from_numpy(lens).cuda()


@pytest.mark.parametrize("kv_name", ["f32", "int8"])
def test_static_scratch_decode_matches_workspace_decode(cuda, kv_name):
    import torch
    import attn_b200 as A
    kv = A.I8 if kv_name == "int8" else A.F32
    shape, q, kc, vc, ks, vs, lens = _case(A, kv, 1000 + kv)
    assert A.decode_workspace_bytes(shape) <= A.STATIC_SCRATCH_BYTES
    # the regular entry point with a caller workspace (not the library's own)
    ws_bytes = A.decode_workspace_bytes(shape)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    ref = torch.empty_like(q)
    A.decode_ex(shape, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), ks.data_ptr() if ks is not None else None,
                vs.data_ptr() if vs is not None else None, lens.data_ptr(), ref.data_ptr(), ws.data_ptr(), ws_bytes)
    torch.cuda.synchronize()
    ref_h = ref.cpu().numpy()
    outs = [torch.full_like(q, float("nan")) for _ in range(2)]
    for i, out in enumerate(outs):                    # two calls in a row share the scratch
        free0 = torch.cuda.mem_get_info()[0]
        A.check(A.lib.attn_decode_static_ex(ctypes.byref(shape), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                            ks.data_ptr() if ks is not None else None,
                                            vs.data_ptr() if vs is not None else None,
                                            lens.data_ptr(), out.data_ptr(), None))
        torch.cuda.synchronize()
        if i == 1:                                    # after the first call has loaded the kernels
            assert torch.cuda.mem_get_info()[0] == free0, "the static entry point took device memory"
        out_h = out.cpu().numpy()
        assert np.isfinite(out_h).all()
        assert rel_err(out_h, ref_h) < F32_TOL


def test_static_scratch_rejects_oversized_shape(cuda):
    import attn_b200 as A
    big = A.DecodeShape(4096, 16, 128, A.F32, 0, 65536, 65536)
    assert A.decode_workspace_bytes(big) > A.STATIC_SCRATCH_BYTES
    st = A.lib.attn_decode_static_ex(ctypes.byref(big), 16, 16, 16, None, None, None, 16, None)
    assert st == A.ERR_WORKSPACE
    assert "scratch" in A.last_error()
