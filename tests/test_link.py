"""The drop-in boundary links (no GPU needed): the reference's own GPU trainer
(train_kaggle.cu + gpu_kernels.cu), with the one edit a maintainer makes --
the reference's attention definitions (gpu_kernels.cu:253-489) inside
#ifndef ATTN_EXTERNAL -- compiles and links against libattn_b200 with the
link line of INTEGRATION.md, and its attn_fwd / attn_bwd then come from the
library.  The edited copy lives in a temporary directory only.  Skipped where
the reference tree is absent."""
import os
import shutil
import subprocess
import sys

import pytest

from conftest import PKG, ROOT

import __graft_entry__ as G

REF = G.REFERENCE_DIR
sys.path.insert(0, os.path.join(ROOT, "tests", "integration"))
import ref_edits  # noqa: E402


def _ref_or_skip():
    if not os.path.exists(os.path.join(REF, "gpu_kernels.cu")):
        pytest.skip("reference tree not present")
    if shutil.which("nvcc") is None:
        pytest.skip("nvcc not present")


def _guarded_copy(dst):
    text = open(os.path.join(REF, "gpu_kernels.cu")).read()
    open(os.path.join(dst, "gpu_kernels.cu"), "w").write(ref_edits.guard_gpu_kernels(text))
    for f in ("gpu_kernels.h", "train_kaggle.cu"):
        shutil.copy(os.path.join(REF, f), dst)


def test_trainer_links_against_the_library(tmp_path):
    _ref_or_skip()
    _guarded_copy(tmp_path)
    exe = tmp_path / "train_gpu"
    cmd = ["nvcc", "-O1", "-arch=sm_100a", "-DATTN_EXTERNAL", "-o", str(exe), "train_kaggle.cu",
           "gpu_kernels.cu", f"-L{PKG}", "-lattn_b200", "-lcublas", f"-Xlinker", f"-rpath={PKG}"]
    r = subprocess.run(cmd, cwd=tmp_path, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    # the trainer's own objects no longer define the attention, and the
    # executable takes attn_fwd / attn_bwd from libattn_b200.so
    undef = subprocess.run(["nm", "-C", "--undefined-only", str(exe)], capture_output=True, text=True).stdout
    assert "attn_fwd(float const*, float const*, float const*, float*, float*)" in undef
    assert "attn_bwd(float*, float*, float*, float*, float const*" in undef
    defined = subprocess.run(["nm", "-C", "--defined-only", str(exe)], capture_output=True, text=True).stdout
    assert "attn_fwd(" not in defined and "k_causal_softmax" not in defined
    needed = subprocess.run(["readelf", "-d", str(exe)], capture_output=True, text=True).stdout
    assert "libattn_b200.so" in needed
    lib_syms = subprocess.run(["nm", "-DC", "--defined-only", os.path.join(PKG, "libattn_b200.so")],
                              capture_output=True, text=True).stdout
    assert "attn_fwd(float const*, float const*, float const*, float*, float*)" in lib_syms


def test_unguarded_trainer_still_builds_on_its_own(tmp_path):
    """Without ATTN_EXTERNAL the edited file is the reference's original."""
    _ref_or_skip()
    _guarded_copy(tmp_path)
    r = subprocess.run(["nvcc", "-O1", "-arch=sm_100a", "-c", "gpu_kernels.cu", "-o", "g.o"], cwd=tmp_path,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    defined = subprocess.run(["nm", "-C", "--defined-only", str(tmp_path / "g.o")], capture_output=True,
                             text=True).stdout
    assert "attn_fwd(float const*" in defined


def test_trainer_with_shrunk_attention_buffers_links(tmp_path):
    _ref_or_skip()
    _guarded_copy(tmp_path)
    # the trainer-side edit that drops the B*H*T*T activation buffers
    src = ref_edits.shrink_trainer(open(tmp_path / "train_kaggle.cu").read())
    open(tmp_path / "train_kaggle.cu", "w").write(src)
    exe = tmp_path / "train_gpu_lse"
    cmd = ["nvcc", "-O1", "-arch=sm_100a", "-DATTN_EXTERNAL", f"-I{os.path.join(ROOT, 'include')}", "-o", str(exe),
           "train_kaggle.cu", "gpu_kernels.cu", f"-L{PKG}", "-lattn_b200", "-lcublas", "-Xlinker", f"-rpath={PKG}"]
    r = subprocess.run(cmd, cwd=tmp_path, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    undef = subprocess.run(["nm", "-C", "--undefined-only", str(exe)], capture_output=True, text=True).stdout
    assert "attn_set_probs_mode" in undef
    assert "attn_fwd(float const*, float const*, float const*, float*, float*)" in undef


def test_trainer_with_fused_qkv_projection_links(tmp_path):
    """On top of the shrunk buffers, the three Q, K, V gemm_nn calls
    (train_kaggle.cu:152-154) replaced by one attn_qkv_proj from the library."""
    _ref_or_skip()
    _guarded_copy(tmp_path)
    src = ref_edits.fuse_qkv(ref_edits.shrink_trainer(open(tmp_path / "train_kaggle.cu").read()))
    assert src.count("attn_qkv_proj(") == 1 and "gemm_nn(a_ln1[l]" not in src
    open(tmp_path / "train_kaggle.cu", "w").write(src)
    exe = tmp_path / "train_gpu_qkv"
    cmd = ["nvcc", "-O1", "-arch=sm_100a", "-DATTN_EXTERNAL", f"-I{os.path.join(ROOT, 'include')}", "-o", str(exe),
           "train_kaggle.cu", "gpu_kernels.cu", f"-L{PKG}", "-lattn_b200", "-lcublas", "-Xlinker", f"-rpath={PKG}"]
    r = subprocess.run(cmd, cwd=tmp_path, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    undef = subprocess.run(["nm", "--undefined-only", str(exe)], capture_output=True, text=True).stdout
    assert " attn_qkv_proj\n" in undef + "\n"
