"""Multi-GPU group logic of the C library, on CPU: the (batch x head) split
plan, and the NCCL-facing host code (group set-up, the watchdog that aborts a
group whose communicator failed, argument checks) run against a fake NCCL
library compiled here, so no GPU and no real communicator is involved."""
import ctypes
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from conftest import PKG, ROOT

import attn_b200 as A

FAKE_NCCL = r"""
#include <stdlib.h>
#include <string.h>
typedef struct { char internal[128]; } ncclUniqueId;
typedef void *ncclComm_t;
static int aborts, destroys, async_err;
static long long gathers;
int fake_aborts(void) { return aborts; }
int fake_destroys(void) { return destroys; }
long long fake_gathers(void) { return gathers; }
void fake_set_async_error(int e) { async_err = e; }
int ncclGetUniqueId(ncclUniqueId *u) { memset(u, 7, sizeof *u); return 0; }
int ncclCommInitRank(ncclComm_t *c, int n, ncclUniqueId u, int r) {
    if (u.internal[0] != 7 || r < 0 || r >= n) return 4;
    *c = malloc(8); return 0; }
int ncclCommInitAll(ncclComm_t *c, int n, const int *devs) {
    for (int i = 0; i < n; i++) c[i] = malloc(8); return 0; }
int ncclCommDestroy(ncclComm_t c) { destroys++; free(c); return 0; }
int ncclCommAbort(ncclComm_t c) { aborts++; free(c); return 0; }
int ncclCommGetAsyncError(ncclComm_t c, int *e) { *e = async_err; return 0; }
int ncclAllGather(const void *s, void *r, unsigned long n, int t, ncclComm_t c, void *st) { gathers++; return 0; }
int ncclGroupStart(void) { return 0; }
int ncclGroupEnd(void) { return 0; }
const char *ncclGetErrorString(int r) { return r ? "fake failure" : "no error"; }
"""


@pytest.fixture(scope="module")
def fake_nccl(tmp_path_factory):
    d = tmp_path_factory.mktemp("fake_nccl")
    src = d / "fake_nccl.c"
    src.write_text(FAKE_NCCL)
    lib = d / "libfake_nccl.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(lib), str(src)], check=True)
    return str(lib)


def run_child(code, env_lib):
    """Runs `code` in a fresh interpreter (one group per process) with the fake NCCL."""
    env = dict(os.environ, ATTN_NCCL_LIB=env_lib, PYTHONPATH=os.pathsep.join([PKG, ROOT]))
    r = subprocess.run([sys.executable, "-c", textwrap.dedent(code)], env=env, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


@pytest.mark.parametrize("B,H", [(8, 16), (4, 16), (2, 12), (1, 16), (3, 8), (6, 4)])
@pytest.mark.parametrize("N", [1, 2, 4, 8])
def test_split_plan_covers_every_unit_once(B, H, N):
    seen = np.zeros((B, H), np.int32)
    try:
        plans = [A.split_plan(B, H, N, r) for r in range(N)]
    except A.AttnError as e:
        assert e.status == A.ERR_UNSUPPORTED
        assert B * H % N or all(B % nb or H % (N // nb) for nb in range(1, N + 1) if N % nb == 0)
        return
    for r, p in enumerate(plans):
        assert p.nb * p.nh == N and B % p.nb == 0 and H % p.nh == 0
        assert p.batch == B // p.nb and p.heads == H // p.nh
        seen[p.batch0:p.batch0 + p.batch, p.head0:p.head0 + p.heads] += 1
        # ranks along the batch first: whole batches when the batch allows it
        if B % N == 0:
            assert p.nh == 1 and p.batch0 == r * (B // N)
    assert (seen == 1).all()


def test_split_plan_rejects_bad_arguments():
    sp = A.Split()
    assert A.lib.attn_split_plan(0, 4, 2, 0, ctypes.byref(sp)) == A.ERR_INVALID
    assert A.lib.attn_split_plan(4, 4, 2, 2, ctypes.byref(sp)) == A.ERR_INVALID
    assert A.lib.attn_split_plan(3, 5, 2, 0, ctypes.byref(sp)) == A.ERR_UNSUPPORTED


def test_gather_workspace_sizes():
    # whole batches: the all-gather writes the output in place, no workspace
    assert A.lib.attn_gather_workspace_bytes(ctypes.byref(A.Shape(8, 16, 1024, 64, 0, 0)), A.BF16, 8) == 0
    # B=4 over 8 ranks: one batch x 8 heads each; local 1024 x 8 x 64 bf16 + 8 such blocks of staging
    local = 1024 * 8 * 64 * 2
    assert A.lib.attn_gather_workspace_bytes(ctypes.byref(A.Shape(4, 16, 1024, 64, 0, 0)), A.BF16, 8) == 9 * local
    assert A.lib.attn_gather_rows_workspace_bytes(8, 4096, 8) == 8 * 4096 * 8


def test_group_calls_need_a_group():
    assert A.lib.attn_group_size() == 0
    assert A.lib.attn_group_sync(None, 0, 10) == A.ERR_INVALID
    assert A.lib.attn_gather_split(ctypes.byref(A.Shape(2, 2, 8, 32, 0, 0)), A.F32, 16, 16, None, 0, None) \
        == A.ERR_INVALID
    assert "attn_init_rank" in A.last_error()


def test_single_process_group_and_watchdog_abort(fake_nccl):
    """attn_init over 4 devices; a communicator reports an asynchronous error;
    attn_group_sync aborts every communicator and removes the group."""
    out = run_child("""
        import ctypes, attn_b200 as A, os
        fake = ctypes.CDLL(os.environ["ATTN_NCCL_LIB"])
        A.check(A.lib.attn_init(4))
        assert A.lib.attn_group_size() == 4
        assert A.lib.attn_init(2) == A.ERR_INVALID          # one group per process
        A.check(A.lib.attn_group_sync(None, 0, 50))         # healthy, nothing in flight
        fake.fake_set_async_error(2)                        # a communicator fails (ncclSystemError)
        st = A.lib.attn_group_sync(None, 0, 50)
        assert st == A.ERR_COMM, st
        assert "aborted" in A.last_error()
        assert fake.fake_aborts() == 4 and fake.fake_destroys() == 0
        assert A.lib.attn_group_size() == 0
        fake.fake_set_async_error(0)
        A.check(A.lib.attn_init(2))                         # a new group after the abort
        A.check(A.lib.attn_finalize())
        assert fake.fake_destroys() == 2 and A.lib.attn_group_size() == 0
        print("ok")
    """, fake_nccl)
    assert "ok" in out


def test_missing_nccl_is_a_clear_error():
    out = run_child("""
        import attn_b200 as A
        st = A.lib.attn_init(2)
        assert st == A.ERR_UNSUPPORTED, st
        assert "cannot load NCCL" in A.last_error()
        print("ok")
    """, "/nonexistent/libnccl.so.2")
    assert "ok" in out


def test_rank_group_from_unique_id(fake_nccl):
    out = run_child("""
        import ctypes, attn_b200 as A
        uid = (ctypes.c_ubyte * 128)()
        A.check(A.lib.attn_get_unique_id(uid))
        assert A.lib.attn_init_rank(2, 2, -1, uid) == A.ERR_INVALID
        A.check(A.lib.attn_init_rank(2, 1, -1, uid))
        assert A.lib.attn_group_size() == 2
        # a single-process entry point refuses a one-process-per-rank group
        assert A.lib.attn_fwd_multi(ctypes.byref(A.Shape(2, 2, 8, 32, 0, 0)), A.F32, None, None, None, None,
                                    None, 0, None, None, None) == A.ERR_INVALID
        A.check(A.lib.attn_finalize())
        print("ok")
    """, fake_nccl)
    assert "ok" in out
