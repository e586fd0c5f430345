"""World-size-2 runs of the multi-GPU host logic on CPU (gloo): every rank
takes its (batch x head) split from the library's attn_split_plan, the
numpy mirror of the gather (all-gather of the compact splits, then the
permute to (B*T, H*d)) must reproduce the single-process result, the LPT
plan for ragged decode must be identical on every rank, and the ranks join
the library's group from one broadcast id (attn_get_unique_id /
attn_init_rank, against a fake NCCL library)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import PKG, ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import shard
    import synth
    from oracle import oracle as O

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        errs = []
        for B, H in ((2, 8), (1, 8)):          # whole batches per rank; heads split across ranks
            T, d = 40, 32
            qa, ka, va = (synth.normal(s, (B * T, H * d), 0, 0.5) for s in (1, 2, 3))
            sp = shard.split(B, H, world, rank)
            loc = [shard.local_inputs(torch.from_numpy(x), sp, T, d).numpy() for x in (qa, ka, va)]
            # this rank's units (the oracle stands in for the GPU kernel here)
            local, _, _ = O.attn_forward(*loc, sp.batch, T, sp.heads, d)
            parts = [torch.zeros_like(torch.from_numpy(local)) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(local))
            plans = [shard.split(B, H, world, r) for r in range(world)]
            full = shard.permute_grid_np(np.stack([p.numpy() for p in parts]), plans, B, T, H, d)
            ref, _, _ = O.attn_forward(qa, ka, va, B, T, H, d)
            errs.append(float(np.abs(full - ref).max()))
        lens = synth.uniform_int(11, 64, 1, 8192)
        ranks, _ = shard.A.shard_lpt(lens, 16, world)
        digest = torch.tensor([int(ranks.astype(np.int64).sum() * 1000003 % 2 ** 31)], dtype=torch.int64)
        gathered = [torch.zeros_like(digest) for _ in range(world)]
        dist.all_gather(gathered, digest)
        same_plan = all(int(g) == int(digest) for g in gathered)
        shard.init_group(rank, world, -1)      # the fake NCCL (ATTN_NCCL_LIB) needs no device
        in_group = shard.A.lib.attn_group_size() == world
        shard.A.check(shard.A.lib.attn_finalize())
        q.put((rank, max(errs), same_plan and in_group))
    finally:
        dist.destroy_process_group()


def test_split_gather_matches_single_process(tmp_path, monkeypatch):
    from test_group import FAKE_NCCL
    import subprocess
    src = tmp_path / "fake_nccl.c"
    src.write_text(FAKE_NCCL)
    lib = tmp_path / "libfake_nccl.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", str(lib), str(src)], check=True)
    monkeypatch.setenv("ATTN_NCCL_LIB", str(lib))
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=60) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, same_plan in results:
        assert err < 1e-6, (rank, err)
        assert same_plan


def test_permute_mirror_layout():
    import shard
    B, T, H, d, world = 1, 3, 8, 2, 4
    plans = [shard.split(B, H, world, r) for r in range(world)]
    staging = np.arange(world * B * T * (H // world) * d, dtype=np.float32).reshape(world, B * T, H // world * d)
    out = shard.permute_grid_np(staging, plans, B, T, H, d)
    for r, p in enumerate(plans):
        assert p.nh == 4 and p.head0 == r * 2
        assert np.array_equal(out[:, p.head0 * d:(p.head0 + p.heads) * d], staging[r])
