"""Multi-GPU partition of the attention work by (batch x head) units.

One process per GPU (torch.distributed supplies ranks and NCCL).  Attention
has no cross-unit exchange, so the compute path needs no collective: each
rank runs the kernels on its own head slice.  Only a caller that needs the
whole output gets one all-gather, into a [world][B][T][H/world][d] staging
buffer, followed by attn_gather_permute into the (B*T, H*d) layout.

The split plans come from the C ABI (attn_shard_range for contiguous head or
unit ranges, attn_shard_lpt for ragged decode units weighted by cache length).
"""
import numpy as np

import attn_b200 as A


def head_range(heads: int, world: int, rank: int):
    """Heads [h0, h1) of this rank; equal slices when world divides heads."""
    return A.shard_range(heads, world, rank)


def permute_staging_np(staging, world, B, T, H, d):
    """numpy mirror of attn_gather_permute: [G][B][T][H/G][d] -> (B*T, H*d)."""
    s = np.asarray(staging).reshape(world, B, T, H // world, d)
    return s.transpose(1, 2, 0, 3, 4).reshape(B * T, H * d)


def forward_head_shard(q, k, v, B, H, T, d, world, rank):
    """Runs this rank's head slice on the GPU; returns the compact (B*T, Hr*d)
    output and lse [B][Hr][T].  q/k/v are this rank's full-width CUDA tensors."""
    import torch
    h0, h1 = head_range(H, world, rank)
    hn = h1 - h0
    out = torch.empty((B * T, hn * d), dtype=q.dtype, device=q.device)
    lse = torch.empty(B * hn * T, dtype=torch.float32, device=q.device)
    shape = A.Shape(B, hn, T, d, q.stride(0), hn * d)
    esz = q.element_size()
    off = h0 * d * esz
    A.fwd_ex(shape, A.BF16 if esz == 2 else A.F32, q.data_ptr() + off, k.data_ptr() + off, v.data_ptr() + off,
             out.data_ptr(), lse.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return out, lse


def gather_heads(local_out, B, H, T, d, world, group=None):
    """All-gathers equal head shards and permutes them to (B*T, H*d)."""
    import torch
    import torch.distributed as dist
    rows, cols = local_out.shape
    staging = torch.empty((world * rows, cols), dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(staging, local_out.contiguous(), group=group)
    if staging.is_cuda:
        return A.gather_permute_t(staging.reshape(-1, d), world, B, T, H, d)
    return torch.from_numpy(permute_staging_np(staging.numpy(), world, B, T, H, d))
