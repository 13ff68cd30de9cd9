"""BucketedGradReducer on the CUDA path, one rank of an NCCL process group.

The gloo tests (tests/test_distributed.py) check the reducer's arithmetic on
two CPU ranks.  This test runs it where the bench runs it: the fused
MHCLiteBlock on a GPU, whose backward produces the gradients inside the fused
autograd functions, the post-accumulate-grad hooks packing them on the
current CUDA stream, NCCL reducing each bucket with its AVG operation on its
own stream, and finish() copying the results back.  With a single rank the
mean over ranks is the gradient itself, so after two steps every .grad must
equal, bit for bit, the gradients of the same steps without the reducer.
"""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.nn as nn

from flash_mhc import MHCLiteBlock
from flash_mhc.distributed import BucketedGradReducer

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _grads_after_two_steps(blk, xs, gs, reducer=None):
    for x, g in zip(xs, gs):
        blk.zero_grad(set_to_none=True)
        blk(x).backward(g)
        if reducer is not None:
            reducer.finish()
    torch.cuda.synchronize()
    return {n: p.grad.clone() for n, p in blk.named_parameters()}


def test_bucketed_reducer_on_the_fused_block_single_rank_nccl():
    T, C = 4096, 512
    torch.manual_seed(7)
    layer = nn.Linear(C, C, bias=False)
    with torch.no_grad():
        layer.weight.normal_(0.0, 0.02)
    blk = MHCLiteBlock(4, C, layer).cuda().to(torch.bfloat16).train()
    gen = torch.Generator(device="cuda").manual_seed(8)
    xs = [torch.randn(T, 4, C, device="cuda", generator=gen).bfloat16().requires_grad_(True)
          for _ in range(2)]
    gs = [torch.randn(T, 4, C, device="cuda", generator=gen).bfloat16() for _ in range(2)]
    assert blk._uses_fused_path(xs[0])
    ref = _grads_after_two_steps(blk, xs, gs)

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    try:
        reducer = BucketedGradReducer(blk)
        assert len(reducer.buckets) == 2  # the wrapped layer, then the block's own
        got = _grads_after_two_steps(blk, xs, gs, reducer)
        reducer.remove()
    finally:
        dist.destroy_process_group()
    for n, t in ref.items():
        assert got[n].dtype == t.dtype
        assert torch.equal(got[n], t), n
