"""Batch-sharded data parallelism for the deformable convolution.

The op is independent per image in its forward and in grad_input /
grad_offset / grad_mask; only grad_weight and grad_bias are sums over the
batch.  So a data-parallel step shards the batch over ranks (one process per
GPU), runs forward / backward locally, and sums the parameter gradients with
one all-reduce (NCCL over NVLink on B200, gloo on CPU ranks in tests).
"""
from __future__ import annotations

from typing import Iterable, List, Optional, Sequence

import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world_size: int) -> slice:
    """Contiguous, balanced slice of `n` items owned by `rank` (the first
    `n % world_size` ranks take one extra item)."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} out of range for world size {world_size}")
    base, extra = divmod(n, world_size)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def shard_batch(tensors: Sequence[Optional[torch.Tensor]], rank: int,
                world_size: int) -> List[Optional[torch.Tensor]]:
    """The rank's shard (dim 0) of every tensor; None stays None."""
    sizes = {t.shape[0] for t in tensors if t is not None}
    if len(sizes) != 1:
        raise ValueError(f"tensors disagree on the batch size: {sorted(sizes)}")
    sl = shard_range(sizes.pop(), rank, world_size)
    return [t[sl] if t is not None else None for t in tensors]


def allreduce_grads(params: Iterable[torch.nn.Parameter], group=None,
                    average: bool = False) -> None:
    """Sum (or average) the gradients of `params` across the process group
    with one flat all-reduce.  Parameters without a gradient contribute
    zeros, so every rank issues the same collective."""
    params = list(params)
    if not params:
        return
    world = dist.get_world_size(group)
    if world == 1:
        return
    ref = params[0]
    flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1)
                      for p in params]).to(ref.device)
    dist.all_reduce(flat, group=group)
    if average:
        flat /= world
    off = 0
    for p in params:
        n = p.numel()
        g = flat[off:off + n].view_as(p)
        if p.grad is None:
            p.grad = g.clone()
        else:
            p.grad.copy_(g)
        off += n
