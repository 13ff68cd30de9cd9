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


class BucketedGradReducer:
    """Data-parallel gradient all-reduce that overlaps the backward pass.

    The parameters of ``module`` are split into buckets (``buckets``: lists of
    parameters, in the order the backward produces them; by default, for an
    ``MHCLiteBlock``, the wrapped layer's parameters first and the block's own
    ``W_all`` / alphas second).  A post-accumulate-grad hook counts each
    bucket's gradients as the backward writes them; once a bucket is complete
    its gradients are packed into a preallocated buffer of ``reduce_dtype``
    (float32 by default) with one multi-tensor copy, and an asynchronous
    all-reduce of that buffer starts.  In the fused block the layer's gradient
    is ready before the K3/K2/K1 backward and the grad_x combination run, so
    its (large) reduction proceeds on NCCL's stream while those kernels
    compute; the block's own gradients (small) are returned with grad_x at the
    end of the backward.  Buckets are launched strictly in bucket order (a bucket
    that completes early waits for the ones before it), so every rank issues
    the same collectives in the same order.

    Call ``finish()`` after ``backward()``: it launches any bucket still
    pending (parameters without a gradient count as zero), makes the current
    stream wait for the reductions and writes the results back into ``.grad``
    with one multi-tensor copy per bucket.  With ``average`` the result is the
    mean over ranks: a SUM all-reduce and a scale, or with ``avg_op`` (NCCL
    only) NCCL's AVG reduction.
    """

    def __init__(self, module: torch.nn.Module, buckets=None, group=None, average: bool = True,
                 reduce_dtype: torch.dtype = torch.float32, avg_op: bool = False):
        self.group = group
        self.average = average
        self.reduce_dtype = reduce_dtype
        if buckets is None:
            buckets = default_buckets(module)
        self.buckets = []
        seen = set()
        for plist in buckets:
            plist = [p for p in plist if p.requires_grad and id(p) not in seen]
            seen.update(id(p) for p in plist)
            if plist:
                self.buckets.append({"params": plist, "ready": 0, "work": None, "buf": None,
                                     "views": None})
        rest = [p for p in module.parameters() if p.requires_grad and id(p) not in seen]
        if rest:
            self.buckets.append({"params": rest, "ready": 0, "work": None, "buf": None,
                                 "views": None})
        self._index = {}
        self._handles = []
        for bi, b in enumerate(self.buckets):
            for p in b["params"]:
                self._index[id(p)] = bi
                self._handles.append(p.register_post_accumulate_grad_hook(self._hook))
        self._next = 0  # first bucket not launched yet
        # avg_op: NCCL averages in the collective itself; otherwise (and on
        # other backends) the buckets are summed and scaled in finish()
        self._avg_in_collective = avg_op and average and dist.get_backend(group) == "nccl"
        self._op = dist.ReduceOp.AVG if self._avg_in_collective else dist.ReduceOp.SUM

    def _buffer(self, b, device):
        if b["buf"] is None:
            total = sum(p.numel() for p in b["params"])
            buf = torch.empty(total, dtype=self.reduce_dtype, device=device)
            views, off = [], 0
            for p in b["params"]:
                views.append(buf[off:off + p.numel()].view(p.shape))
                off += p.numel()
            b["buf"], b["views"] = buf, views
        return b["buf"]

    def _launch(self, b):
        params = b["params"]
        dev = next((p.grad.device for p in params if p.grad is not None), params[0].device)
        buf = self._buffer(b, dev)
        have = [(v, p.grad) for v, p in zip(b["views"], params) if p.grad is not None]
        if len(have) < len(params):
            buf.zero_()
        if have:
            torch._foreach_copy_([v for v, _ in have], [g for _, g in have])
        b["work"] = dist.all_reduce(buf, op=self._op, group=self.group, async_op=True)

    def _launch_ready(self):
        while self._next < len(self.buckets):
            b = self.buckets[self._next]
            if b["ready"] < len(b["params"]):
                return
            self._launch(b)
            self._next += 1

    def _hook(self, p):
        self.buckets[self._index[id(p)]]["ready"] += 1
        self._launch_ready()

    def finish(self) -> None:
        for b in self.buckets[self._next:]:
            b["ready"] = len(b["params"])
        self._launch_ready()
        world = dist.get_world_size(self.group)
        for b in self.buckets:
            b["work"].wait()
            if self.average and world > 1 and not self._avg_in_collective:
                b["buf"].mul_(1.0 / world)
            grads = []
            for p, v in zip(b["params"], b["views"]):
                if p.grad is None:
                    p.grad = torch.empty_like(p)
                grads.append(p.grad)
            torch._foreach_copy_(grads, b["views"])
            b["ready"], b["work"] = 0, None
        self._next = 0

    def remove(self) -> None:
        """Unregister the hooks."""
        for h in self._handles:
            h.remove()
        self._handles = []


def default_buckets(module: torch.nn.Module) -> list:
    """Buckets in backward order for an ``MHCLiteBlock``: the wrapped layer's
    parameters (their gradients are ready after the layer's backward), then the
    block's own parameters (ready after the K2 and K1 backward).  Any other
    module: one bucket of all its parameters."""
    layer = getattr(module, "layer", None)
    if isinstance(layer, torch.nn.Module):
        lp = [p for p in layer.parameters() if p.requires_grad]
        lids = {id(p) for p in lp}
        own = [p for p in module.parameters() if p.requires_grad and id(p) not in lids]
        return [lp, own]
    return [[p for p in module.parameters() if p.requires_grad]]
