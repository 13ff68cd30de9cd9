"""Token-sharded data parallelism on CPU with gloo (world_size 2).

* shard_bounds/shard_tokens partition T exactly;
* every rank runs MHCLiteBlock on its token shard (pure-PyTorch path on CPU,
  the same math the fused CUDA path restates) and allreduce_gradients sums the
  parameter gradients in one bucket: the result equals the single-process
  full-batch gradient (the path's only exchange); BucketedGradReducer does the
  same per bucket from post-accumulate-grad hooks during the backward;
* failure detection on the host: a rank that dies before the collective makes
  the surviving rank's all-reduce fail after the process-group timeout instead
  of hanging.
"""

from __future__ import annotations

import os
import socket
import tempfile
import traceback
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

from flash_mhc import MHCLiteBlock
from flash_mhc.distributed import (BucketedGradReducer, allreduce_gradients, shard_bounds,
                                   shard_tokens)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_bounds_partition_exactly():
    for T in (0, 1, 7, 64, 65537):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(T, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == T
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    x = torch.arange(10)
    assert torch.equal(torch.cat([shard_tokens(x, r, 3) for r in range(3)]), x)
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def _model(seed):
    torch.manual_seed(seed)
    C = 16
    layer = nn.Linear(C, C, bias=False)
    blk = MHCLiteBlock(4, C, layer)
    with torch.no_grad():
        blk.alpha_pre.fill_(0.5)
        blk.alpha_post.fill_(0.7)
        blk.alpha_res.fill_(0.9)
    return blk


def _data(T=37, C=16):
    g = torch.Generator().manual_seed(123)
    return torch.randn(T, 4, C, generator=g), torch.randn(T, 4, C, generator=g)


def _worker(rank, world, port, out_dir, mode):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=10 if mode == "fail" else 60))
        if mode == "fail":
            if rank == 1:
                os._exit(3)  # dies without joining the collective
            try:
                dist.all_reduce(torch.ones(4))
                result = "no error"
            except Exception as e:  # expected: the peer is gone
                result = f"error: {type(e).__name__}"
            torch.save({"result": result}, os.path.join(out_dir, f"r{rank}.pt"))
            os._exit(0)
        blk = _model(0)
        x, g = _data()
        xs, gs = shard_tokens(x, rank, world), shard_tokens(g, rank, world)
        if mode == "bucketed_unused":
            # a layer parameter the forward never uses gets no gradient: the
            # layer bucket cannot complete in the hooks, so the block's own
            # bucket (complete during backward) must wait for it, and finish()
            # launches both in bucket order with zeros for the unused one
            blk.layer.register_parameter("unused", nn.Parameter(torch.ones(3)))
            red = BucketedGradReducer(blk)
            (blk(xs) * gs).sum().backward()
            assert red._next == 0  # nothing launched: the first bucket is incomplete
            red.finish()
            red.remove()
            grads = {n: p.grad.clone() for n, p in blk.named_parameters()}
            torch.save({"grads": grads}, os.path.join(out_dir, f"r{rank}.pt"))
            dist.barrier()
            dist.destroy_process_group()
            return
        if mode == "bucketed":
            # two steps through the overlapped reducer: the hooks launch each
            # bucket during backward; the second step checks the state resets
            red = BucketedGradReducer(blk)
            assert len(red.buckets) == 2  # the wrapped layer, then the block's own
            for _ in range(2):
                blk.zero_grad(set_to_none=True)
                (blk(xs) * gs).sum().backward()
                red.finish()
            red.remove()
            grads = {n: p.grad.clone() for n, p in blk.named_parameters()}
            torch.save({"grads": grads}, os.path.join(out_dir, f"r{rank}.pt"))
            dist.barrier()
            dist.destroy_process_group()
            return
        out = blk(xs)
        (out * gs).sum().backward()
        if mode == "async":
            work, finish = allreduce_gradients(blk, average=False, async_op=True)
            work.wait()
            finish()
        else:
            allreduce_gradients(blk, average=(mode == "avg"))
        grads = {n: p.grad.clone() for n, p in blk.named_parameters()}
        torch.save({"grads": grads}, os.path.join(out_dir, f"r{rank}.pt"))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


def _run(mode, world=2):
    out_dir = tempfile.mkdtemp(prefix="fmhc_dist_")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out_dir, mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            p.join()
    errs = [f for f in os.listdir(out_dir) if f.startswith("err")]
    assert not errs, open(os.path.join(out_dir, errs[0])).read()
    return out_dir, procs


def _reference_grads():
    blk = _model(0)
    x, g = _data()
    (blk(x) * g).sum().backward()
    return {n: p.grad.clone() for n, p in blk.named_parameters()}


@pytest.mark.parametrize("mode", ["sum", "async", "avg", "bucketed", "bucketed_unused"])
def test_token_sharded_grads_equal_full_batch(mode):
    out_dir, procs = _run(mode)
    assert all(p.exitcode == 0 for p in procs)
    ref = _reference_grads()
    scale = 0.5 if mode in ("avg", "bucketed", "bucketed_unused") else 1.0
    for r in range(2):
        got = torch.load(os.path.join(out_dir, f"r{r}.pt"))["grads"]
        if mode == "bucketed_unused":
            assert torch.equal(got["layer.unused"], torch.zeros(3))
        for n, t in ref.items():
            torch.testing.assert_close(got[n], t * scale, atol=1e-5, rtol=1e-4, msg=n)


def test_dead_rank_makes_collective_fail_not_hang():
    out_dir, procs = _run("fail")
    assert procs[1].exitcode == 3
    res = torch.load(os.path.join(out_dir, "r0.pt"))["result"]
    assert res.startswith("error"), res
