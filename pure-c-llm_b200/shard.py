"""Python client of the library's multi-GPU entry points (one process per GPU).

The split and the gathers live in the C library (csrc/group.cu):
attn_split_plan says which (batch x head) units a rank computes,
attn_shard_lpt balances ragged decode sequences, attn_init_rank joins the
library's own NCCL communicator, and attn_gather_split / attn_gather_rows
assemble whole outputs.  This module only moves the 128-byte communicator id
between ranks (over whatever torch.distributed group the caller already
has) and wraps tensors as pointers for the tests and the benchmark.
"""
import ctypes

import numpy as np

import attn_b200 as A


def split(B: int, H: int, world: int, rank: int) -> A.Split:
    return A.split_plan(B, H, world, rank)


def init_group(rank: int, world: int, device: int):
    """Joins the library's NCCL group: rank 0 makes the id, torch.distributed
    broadcasts it (any backend), every rank calls attn_init_rank."""
    import torch
    import torch.distributed as dist
    uid = (ctypes.c_ubyte * 128)()
    if rank == 0:
        A.check(A.lib.attn_get_unique_id(uid))
    backend = dist.get_backend()
    t = torch.tensor(list(bytes(uid)), dtype=torch.uint8,
                     device=f"cuda:{device}" if backend == "nccl" else "cpu")
    dist.broadcast(t, 0)
    uid = (ctypes.c_ubyte * 128)(*t.cpu().tolist())
    A.check(A.lib.attn_init_rank(world, rank, device, uid))


def local_inputs(full, sp: A.Split, T: int, d: int):
    """This rank's compact (batch*T, heads*d) slice of a full (B*T, H*d) tensor."""
    rows = slice(sp.batch0 * T, (sp.batch0 + sp.batch) * T)
    cols = slice(sp.head0 * d, (sp.head0 + sp.heads) * d)
    return full[rows, cols].contiguous()


def gather_split(local, B: int, H: int, T: int, d: int, out=None, stream=None):
    """Whole (B*T, H*d) output on every rank from each rank's compact split."""
    import torch
    dt = A.BF16 if local.dtype == torch.bfloat16 else A.F32
    shape = A.Shape(B, H, T, d, 0, 0)
    out = torch.empty((B * T, H * d), dtype=local.dtype, device=local.device) if out is None else out
    nbytes = A.lib.attn_gather_workspace_bytes(ctypes.byref(shape), dt, A.lib.attn_group_size())
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=local.device)
    s = torch.cuda.current_stream().cuda_stream if stream is None else stream
    A.check(A.lib.attn_gather_split(ctypes.byref(shape), dt, local.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                    nbytes, s))
    return out


def permute_grid_np(staging, plans, B, T, H, d):
    """numpy mirror of the gather's permute: staging [nranks][batch*T][heads*d]
    (rank r's compact split) -> (B*T, H*d)."""
    out = np.empty((B * T, H * d), dtype=staging.dtype)
    for r, p in enumerate(plans):
        out[p.batch0 * T:(p.batch0 + p.batch) * T, p.head0 * d:(p.head0 + p.heads) * d] = staging[r]
    return out


def lpt_sequences(lens, world: int):
    """Sequences per rank (attn_shard_lpt with one unit per sequence)."""
    ranks, load = A.shard_lpt(lens, 1, world)
    return [np.flatnonzero(ranks == r) for r in range(world)], load
