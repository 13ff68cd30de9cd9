"""Token-sharded data parallelism for mHC-lite blocks.

Every mHC-lite op is token-local, so a batch of T tokens splits into
contiguous per-rank shards with no communication in the forward pass.  The
only cross-token quantities are parameter gradients (W_all.weight/bias, the
three alphas, and the wrapped layer's own parameters); ``allreduce_gradients``
sums them across ranks in one flat float32 bucket (a single NCCL all-reduce
over NVLink on GPUs, gloo on CPU) and scales by 1/world_size so the result
equals the gradient of the mean loss over the global batch when each rank's
loss is the mean over its own shard.

The reference library is single-GPU and has no distributed code; this module
is the data-parallel layer the B200 build adds around it.
"""

from __future__ import annotations

from typing import Iterable

import torch
import torch.distributed as dist


def shard_bounds(T: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous token shard; sizes differ by at most 1."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world {rank}/{world}")
    base, rem = divmod(T, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def shard_tokens(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank's contiguous slice of the token dimension (dim 0) of ``x``."""
    s, e = shard_bounds(x.shape[0], rank, world)
    return x[s:e]


def flatten_grads(params: Iterable[torch.nn.Parameter], device=None) -> tuple[torch.Tensor, list]:
    """Concatenate the grads of ``params`` (missing grads count as zero) into one f32 bucket."""
    plist = [p for p in params if p.requires_grad]
    if not plist:
        return torch.zeros(0, dtype=torch.float32, device=device), []
    dev = device or plist[0].device
    total = sum(p.numel() for p in plist)
    bucket = torch.empty(total, dtype=torch.float32, device=dev)
    off = 0
    for p in plist:
        n = p.numel()
        if p.grad is None:
            bucket[off:off + n].zero_()
        else:
            bucket[off:off + n].copy_(p.grad.reshape(-1))
        off += n
    return bucket, plist


def unflatten_grads(bucket: torch.Tensor, plist: list) -> None:
    off = 0
    for p in plist:
        n = p.numel()
        g = bucket[off:off + n].view_as(p).to(p.dtype)
        if p.grad is None:
            p.grad = g.clone()
        else:
            p.grad.copy_(g)
        off += n


def allreduce_gradients(module: torch.nn.Module, group=None, average: bool = True,
                        async_op: bool = False):
    """All-reduce every parameter gradient of ``module`` in one flat f32 bucket.

    With ``async_op=True`` returns ``(work, finish)``: call ``work.wait()`` (or
    let the stream order it) and then ``finish()`` to scatter the reduced bucket
    back into ``.grad``.  Otherwise reduces in place and returns None.
    """
    world = dist.get_world_size(group)
    bucket, plist = flatten_grads(module.parameters())
    if not plist:
        return None
    work = dist.all_reduce(bucket, op=dist.ReduceOp.SUM, group=group, async_op=async_op)

    def finish():
        if average and world > 1:
            bucket.div_(world)
        unflatten_grads(bucket, plist)

    if async_op:
        return work, finish
    finish()
    return None
