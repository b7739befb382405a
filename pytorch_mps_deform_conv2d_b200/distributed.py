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


def _adjacent_view(grads: Sequence[Optional[torch.Tensor]]) -> Optional[torch.Tensor]:
    """One 1-D view covering `grads` when they are contiguous and lie back to
    back in one storage, in any order of the list (a GradBucket lays them out
    that way, and so does the operator's autograd node for grad_weight and
    grad_bias); None otherwise."""
    if not grads or any(g is None or not g.is_contiguous() for g in grads):
        return None
    grads = sorted(grads, key=lambda g: g.data_ptr())
    first = grads[0]
    storage = first.untyped_storage()
    end = first.data_ptr()
    for g in grads:
        if (g.dtype != first.dtype or g.device != first.device
                or g.untyped_storage().data_ptr() != storage.data_ptr() or g.data_ptr() != end):
            return None
        end += g.numel() * g.element_size()
    total = sum(g.numel() for g in grads)
    return first.new_empty(0).set_(storage, first.storage_offset(), (total,), (1,))


def allreduce_grads(params: Iterable[torch.nn.Parameter], group=None,
                    average: bool = False) -> None:
    """Sum (or average) the gradients of `params` across the process group.

    The gradients are reduced where they lie, without packing copies: in one
    all-reduce when they sit back to back in one buffer, else as one
    all-reduce per gradient issued together in a single collective group
    (NCCL runs them as one launch; other backends back to back).  Parameters without a gradient get a zero
    gradient first, so every rank issues the same collectives."""
    params = list(params)
    if not params:
        return
    world = dist.get_world_size(group)
    if world == 1:
        return
    for p in params:
        if p.grad is None:
            p.grad = torch.zeros_like(p)
    grads = [p.grad for p in params]
    flat = _adjacent_view(grads)
    if flat is not None:
        dist.all_reduce(flat, group=group)
    elif dist.get_backend(group) == "nccl":
        with dist._coalescing_manager(group=group, device=grads[0].device):
            for g in grads:
                dist.all_reduce(g, group=group)
    else:  # backends without coalescing (gloo): the collectives back to back
        for work in [dist.all_reduce(g, group=group, async_op=True) for g in grads]:
            work.wait()
    if average:
        for g in grads:
            g /= world


class GradBucket:
    """The gradients of `params` as views of one flat buffer (a data-parallel
    gradient bucket): ``zero_()`` clears them for the next step, autograd
    then accumulates each parameter's gradient into its view in place, and
    :func:`allreduce_grads` sums the whole bucket with one all-reduce (on 8
    B200s, 35 us for a DCN layer's 2.36 MB against 53 us for its two
    gradients as one coalesced group).  Keep ``p.grad`` as set here: do not
    assign ``None`` to it between steps."""

    def __init__(self, params: Iterable[torch.nn.Parameter]):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("no parameters that require a gradient")
        dtypes = {p.dtype for p in self.params}
        devices = {p.device for p in self.params}
        if len(dtypes) != 1 or len(devices) != 1:
            raise ValueError("a bucket holds gradients of one dtype on one device")
        self.flat = torch.zeros(sum(p.numel() for p in self.params),
                                dtype=self.params[0].dtype, device=self.params[0].device)
        offset = 0
        for p in self.params:
            p.grad = self.flat[offset:offset + p.numel()].view_as(p)
            offset += p.numel()

    def zero_(self) -> None:
        self.flat.zero_()


class GradAllReduce:
    """Sums `params`' gradients across the group as soon as the backward has
    produced them, the way a data-parallel wrapper does: a hook on each
    parameter (``register_post_accumulate_grad_hook``) counts the gradients
    accumulated in this backward, and when the last of them is in, one
    asynchronous collective (one coalesced NCCL group; gloo: back-to-back
    async all-reduces) starts on them while autograd goes on with the layers
    before this one.  ``wait()`` -- before the optimizer step -- blocks until
    it is done (with ``average``, divides by the world size) and re-arms the
    hooks for the next step.  Every rank must run the same backward, so the
    collectives match; a parameter that got no gradient in a step has none
    reduced (call ``wait()`` on every rank all the same).  One backward per
    step: with gradients accumulated over several backward passes, the
    collective would start after the first of them -- reduce with
    :func:`allreduce_grads` after the last one instead.

        sync = GradAllReduce(module.parameters())
        loss.backward()
        sync.wait()
        opt.step()
    """

    def __init__(self, params: Iterable[torch.nn.Parameter], group=None,
                 average: bool = False):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.average = average
        self._ready: List[torch.nn.Parameter] = []
        self._works = []
        self._handles = [p.register_post_accumulate_grad_hook(self._on_grad)
                         for p in self.params]

    def _on_grad(self, p: torch.nn.Parameter) -> None:
        self._ready.append(p)
        if len(self._ready) == len(self.params):
            self._launch()

    def _launch(self) -> None:
        grads = [p.grad for p in self._ready]
        if dist.get_world_size(self.group) == 1:
            return
        flat = _adjacent_view(grads)
        if flat is not None:  # a GradBucket's views: one collective
            self._works = [dist.all_reduce(flat, group=self.group, async_op=True)]
        elif dist.get_backend(self.group) == "nccl":
            with dist._coalescing_manager(group=self.group, device=grads[0].device,
                                          async_ops=True) as cm:
                for g in grads:
                    dist.all_reduce(g, group=self.group)
            self._works = [cm]
        else:
            self._works = [dist.all_reduce(g, group=self.group, async_op=True) for g in grads]

    def wait(self) -> None:
        """Waits for this step's collective (launching it for the gradients
        that did arrive, if not all parameters got one) and re-arms."""
        if self._ready and not self._works and len(self._ready) < len(self.params):
            self._launch()
        for w in self._works:
            w.wait()
        if self.average and self._ready:
            world = dist.get_world_size(self.group)
            for p in self._ready:
                p.grad /= world
        self._ready, self._works = [], []

    def remove(self) -> None:
        """Detaches the hooks."""
        for h in self._handles:
            h.remove()
        self._handles = []


# ---------------------------------------------------------------------------
# Row slabs: more ranks than images
# ---------------------------------------------------------------------------
# With more ranks than images, each image's output rows are split into slabs
# over the ranks that share it.  The input is replicated on those ranks (the
# offsets are unbounded, so there is no fixed halo); each rank computes its
# slab's rows and the gradients of its slab: grad_offset / grad_mask of its
# rows (owned, no exchange) and its contributions to grad_input (summed over
# the image's ranks) and to grad_weight / grad_bias (summed over all ranks).

def image_slab(rank: int, world_size: int, n_images: int):
    """(first image, image count, slab, slabs per image) of `rank`: batch
    sharding when world_size <= n_images (slabs per image 1), else
    world_size / n_images slabs of each image (world_size must then be a
    multiple of n_images)."""
    if world_size <= n_images:
        sl = shard_range(n_images, rank, world_size)
        return sl.start, sl.stop - sl.start, 0, 1
    if world_size % n_images:
        raise ValueError(f"{world_size} ranks cannot split {n_images} images evenly")
    slabs = world_size // n_images
    return rank // slabs, 1, rank % slabs, slabs


def slab_rows(out_h: int, slab: int, slabs: int) -> slice:
    """Output rows of slab `slab` of `slabs` balanced slabs."""
    return shard_range(out_h, slab, slabs)


def image_groups(world_size: int, n_images: int):
    """One process group per image shared by several ranks (created on
    every rank, in the same order); [] when no image is shared."""
    _, _, _, slabs = image_slab(0, world_size, n_images)
    if slabs == 1:
        return []
    return [dist.new_group(list(range(i * slabs, (i + 1) * slabs))) for i in range(n_images)]


class _SumGradOver(torch.autograd.Function):
    """Identity forward; the gradient is summed over `group` (an all-reduce)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, grad):
        grad = grad.contiguous()
        if ctx.group is not None:
            dist.all_reduce(grad, group=ctx.group)
        return grad, None


def deform_conv2d_row_sharded(input, offset_rows, weight, bias=None, stride=(1, 1),
                              padding=(0, 0), dilation=(1, 1), mask_rows=None,
                              row_begin: int = 0, group=None, flags=None):
    """This rank's output rows ``[row_begin, row_begin + offset_rows.shape[2])``
    of the deformable convolution of a replicated ``input``; in the backward
    the input's gradient is summed over ``group`` (the ranks holding the other
    rows of the same images).  grad_weight / grad_bias stay per rank: sum them
    with :func:`allreduce_grads` as in batch data parallelism."""
    from .ops import deform_conv2d_rows
    x = _SumGradOver.apply(input, group) if group is not None else input
    return deform_conv2d_rows(x, offset_rows, weight, bias, stride, padding, dilation, mask_rows,
                              row_begin=row_begin, flags=flags)
