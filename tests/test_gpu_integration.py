"""The reference's decoder block with its attention on the GPU.

tests/integration/ builds transformer.c's forward_block (transformer.c:251-285)
twice from the reference sources: unmodified (block_ref, the CPU reference)
and with its attention call routed to attn_cached_attention_host (block_gpu,
the maintainer's one-line edit).  Both run 16 layers x 128 tokens at the C1
decode shape (d_model 512 = 16 x 32, 512 cached rows before the first token)
from the same seed; every token's residual vector and last attention output
must agree within the fp32 tolerance.  The programs are prebuilt, so this
test needs the GPU and not the reference tree."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu
BUILD = os.path.join(ROOT, "tests", "integration", "_build")
F32_TOL = 1e-5


def test_forward_block_routed_to_gpu_matches_reference(cuda, tmp_path):
    ref, gpu = os.path.join(BUILD, "block_ref"), os.path.join(BUILD, "block_gpu")
    if not (os.path.exists(ref) and os.path.exists(gpu)):
        pytest.skip("integration programs not built (the reference tree was absent at build time)")
    env = dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count() or 1))
    outs = {}
    for name, exe in (("ref", ref), ("gpu", gpu)):
        path = tmp_path / f"{name}.bin"
        r = subprocess.run([exe, str(path)], env=env, capture_output=True, text=True, timeout=600)
        assert r.returncode == 0, r.stderr
        outs[name] = np.fromfile(path, dtype=np.float32).reshape(128, 2, 512)
    for which in (0, 1):               # residual vector, last layer's attention output
        a, b = outs["gpu"][:, which].astype(np.float64), outs["ref"][:, which].astype(np.float64)
        err = np.abs(a - b).max(axis=1) / np.maximum(np.abs(b).max(axis=1), 1e-6)
        assert err.max() < F32_TOL, (which, err.max(), int(err.argmax()))
