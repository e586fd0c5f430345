"""The head-sharded multi-GPU forward on real GPUs (NCCL): every rank runs the
tensor-core kernel on its head slice, the outputs are all-gathered into the
[world][B][T][H/world][d] staging layout and permuted back with
attn_gather_permute.  The result must equal the single-GPU forward bit for
bit (each (batch, head) unit is computed identically wherever it runs).
Skipped when fewer than two GPUs are visible."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import PKG, ROOT

pytestmark = pytest.mark.gpu


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
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import attn_b200 as A
    import shard

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        res = {}
        for name, dt in (("bf16", torch.bfloat16), ("f32", torch.float32)):
            B, H, T, d = 2, 8, 384, 64
            g = torch.Generator(device=dev).manual_seed(7)
            qkv = [(torch.randn((B * T, H * d), generator=g, device=dev) * 0.5).to(dt) for _ in range(3)]
            local, _ = shard.forward_head_shard(*qkv, B, H, T, d, world, rank)
            full = shard.gather_heads(local, B, H, T, d, world)
            ref, _ = A.forward_t(*qkv, H, B)
            torch.cuda.synchronize()
            res[name] = bool(torch.equal(full, ref))
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_head_sharded_forward_gathers_to_single_gpu_result(cuda):
    import torch
    world = min(2, torch.cuda.device_count())
    if world < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, res in results:
        assert res == {"bf16": True, "f32": True}, (rank, res)
