"""The multi-GPU split on real GPUs, through the library's own NCCL group.

* One process per GPU (attn_init_rank): each rank runs the forward on its
  (batch x head) split from attn_split_plan and attn_gather_split assembles
  the whole output on every rank; the result must equal the single-GPU
  forward bit for bit (a unit is computed identically wherever it runs).
  Ragged decode: sequences are dealt by attn_shard_lpt, each rank decodes its
  own, and attn_gather_rows puts every row in place.
* One process driving both GPUs (attn_init + attn_fwd_multi /
  attn_decode_multi), the reference trainer's single-process model.

NVLS is off; no kernel reads another GPU's memory.  Skipped when fewer than
two GPUs are visible."""
import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import PKG, ROOT

pytestmark = pytest.mark.gpu
F32_TOL = 1e-5


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
    import synth

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    res = {}
    try:
        shard.init_group(rank, world, rank)
        for B, H in ((2, 8), (1, 8)):                  # whole batches; heads split across ranks
            for name, dt in (("bf16", torch.bfloat16), ("f32", torch.float32)):
                T, d = 384, 64
                g = torch.Generator(device=dev).manual_seed(7)
                qkv = [(torch.randn((B * T, H * d), generator=g, device=dev) * 0.5).to(dt) for _ in range(3)]
                sp = shard.split(B, H, world, rank)
                loc = [shard.local_inputs(x, sp, T, d) for x in qkv]
                local, _ = A.forward_t(*loc, sp.heads, sp.batch)
                full = shard.gather_split(local, B, H, T, d)
                ref, _ = A.forward_t(*qkv, H, B)
                torch.cuda.synchronize()
                res[f"fwd_B{B}_{name}"] = bool(torch.equal(full, ref))
        # ragged decode: LPT over sequences, local caches, gathered rows
        n, H, d, max_len = 12, 16, 64, 3000
        lens = synth.uniform_int(5, n, 1, max_len)
        seqs, _ = shard.lpt_sequences(lens, world)
        mine = seqs[rank]
        max_local = max(len(s) for s in seqs)
        g = torch.Generator(device=dev).manual_seed(11)
        kc = torch.randn((n * max_len, H * d), generator=g, device=dev)
        vc = torch.randn((n * max_len, H * d), generator=g, device=dev)
        qa = torch.randn((n, H * d), generator=g, device=dev)
        lens_d = torch.from_numpy(lens).to(dev)
        idx = torch.from_numpy(mine).to(dev)
        kl = kc.view(n, max_len, H * d)[idx].reshape(-1, H * d).contiguous()
        vl = vc.view(n, max_len, H * d)[idx].reshape(-1, H * d).contiguous()
        out_local = torch.zeros((max_local, H * d), device=dev)
        if len(mine):
            A.decode_t(qa[idx].contiguous(), kl, vl, lens_d[idx].contiguous(), H, max_len, max_len,
                       out=out_local[:len(mine)])
        order = np.full((world, max_local), -1, np.int32)
        for r, s in enumerate(seqs):
            order[r, :len(s)] = s
        order_d = torch.from_numpy(order.reshape(-1)).to(dev)
        out = torch.zeros((n, H * d), device=dev)
        row_bytes = H * d * 4
        nbytes = A.lib.attn_gather_rows_workspace_bytes(max_local, row_bytes, world)
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        A.check(A.lib.attn_gather_rows(out_local.data_ptr(), max_local, row_bytes, order_d.data_ptr(), n,
                                       out.data_ptr(), ws.data_ptr(), nbytes,
                                       torch.cuda.current_stream().cuda_stream))
        ref = A.decode_t(qa, kc, vc, lens_d, H, max_len, max_len)
        torch.cuda.synchronize()
        err = float(((out - ref).abs().max() / ref.abs().max()).item())
        res["decode_gather"] = err < F32_TOL
        torch.cuda.synchronize()
        A.check(A.lib.attn_finalize())
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_rank_split_gathers_to_single_gpu_result(cuda):
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
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, res in results:
        assert res and all(res.values()), (rank, res)


SINGLE_PROCESS = r"""
import ctypes, numpy as np, torch
import attn_b200 as A, synth
G = 2
A.check(A.lib.attn_init(G))
P = ctypes.c_void_p
def arr(xs, t=P):
    return (t * len(xs))(*xs)
ok = {}
for B, H in ((2, 8), (1, 8)):
    T, d = 256, 64
    g = torch.Generator().manual_seed(3)
    host = [(torch.randn((B * T, H * d), generator=g) * 0.5).to(torch.bfloat16) for _ in range(3)]
    qkv = [[x.to(f"cuda:{i}") for x in host] for i in range(G)]
    outs = [torch.zeros((B * T, H * d), dtype=torch.bfloat16, device=f"cuda:{i}") for i in range(G)]
    shape = A.Shape(B, H, T, d, 0, 0)
    nb = A.lib.attn_gather_workspace_bytes(ctypes.byref(shape), A.BF16, G)
    ws = [torch.empty(max(nb, 256), dtype=torch.uint8, device=f"cuda:{i}") for i in range(G)]
    streams = [torch.cuda.Stream(device=i) for i in range(G)]
    A.check(A.lib.attn_fwd_multi(ctypes.byref(shape), A.BF16, arr([qkv[i][0].data_ptr() for i in range(G)]),
                                 arr([qkv[i][1].data_ptr() for i in range(G)]),
                                 arr([qkv[i][2].data_ptr() for i in range(G)]), arr([o.data_ptr() for o in outs]),
                                 None, 1, arr([w.data_ptr() for w in ws]), arr([nb] * G, ctypes.c_size_t),
                                 arr([s.cuda_stream for s in streams])))
    A.check(A.lib.attn_group_sync(arr([s.cuda_stream for s in streams]), G, 30000))
    with torch.cuda.device(0):
        ref, _ = A.forward_t(*qkv[0], H, B)
    torch.cuda.synchronize(0)
    ok[f"fwd_B{B}"] = all(torch.equal(o.cpu(), ref.cpu()) for o in outs)
# decode: device i holds sequences i, i+2, ...
n, H, d, max_len = 7, 16, 32, 900
lens = synth.uniform_int(9, n, 1, max_len)
g = torch.Generator().manual_seed(4)
kc, vc, qa = (torch.randn((n * max_len, H * d), generator=g), torch.randn((n * max_len, H * d), generator=g),
              torch.randn((n, H * d), generator=g))
seqs = [np.arange(i, n, G) for i in range(G)]
max_local = max(len(s) for s in seqs)
dv = []
for i, s in enumerate(seqs):
    dd = f"cuda:{i}"
    idx = torch.from_numpy(s)
    dv.append(dict(q=qa[idx].contiguous().to(dd), k=kc.view(n, max_len, -1)[idx].reshape(-1, H * d).contiguous().to(dd),
                   v=vc.view(n, max_len, -1)[idx].reshape(-1, H * d).contiguous().to(dd),
                   lens=torch.from_numpy(lens[s]).to(dd), out=torch.zeros((max_local, H * d), device=dd),
                   full=torch.zeros((n, H * d), device=dd)))
order = np.full((G, max_local), -1, np.int32)
for i, s in enumerate(seqs):
    order[i, :len(s)] = s
orders = [torch.from_numpy(order.reshape(-1)).to(f"cuda:{i}") for i in range(G)]
shapes = (A.DecodeShape * G)(*[A.DecodeShape(len(s), H, d, A.F32, 0, max_len, max_len) for s in seqs])
nb = A.lib.attn_gather_rows_workspace_bytes(max_local, H * d * 4, G)
ws = [torch.empty(max(nb, 256), dtype=torch.uint8, device=f"cuda:{i}") for i in range(G)]
streams = [torch.cuda.Stream(device=i) for i in range(G)]
A.check(A.lib.attn_decode_multi(shapes, arr([x["q"].data_ptr() for x in dv]), arr([x["k"].data_ptr() for x in dv]),
                                arr([x["v"].data_ptr() for x in dv]), None, None,
                                arr([x["lens"].data_ptr() for x in dv]), arr([x["out"].data_ptr() for x in dv]),
                                1, max_local, arr([o.data_ptr() for o in orders]), n,
                                arr([x["full"].data_ptr() for x in dv]), arr([w.data_ptr() for w in ws]),
                                arr([nb] * G, ctypes.c_size_t), arr([s.cuda_stream for s in streams])))
A.check(A.lib.attn_group_sync(arr([s.cuda_stream for s in streams]), G, 30000))
with torch.cuda.device(0):
    ref = A.decode_t(qa.cuda(0), kc.cuda(0), vc.cuda(0), torch.from_numpy(lens).cuda(0), H, max_len, max_len)
torch.cuda.synchronize(0)
ok["decode"] = all(float((x["full"].cpu() - ref.cpu()).abs().max() / ref.abs().max()) < 1e-5 for x in dv)
A.check(A.lib.attn_finalize())
print("RESULT", ok)
assert all(ok.values()), ok
"""


def test_single_process_group_over_two_gpus(cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=os.pathsep.join([PKG, ROOT]))
    r = subprocess.run([sys.executable, "-c", SINGLE_PROCESS], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
