"""CUDA-graph capture of the fused path (small-T / strong-scaling use).

Every C-ABI call launches on the current stream and does its one-time set-up
(shared-memory opt-in, driver entry points) on the first, eager call, so the
op-level hot path and MHCLiteBlock's fused forward+backward can be captured;
replays must reproduce eager results bit for bit (the kernels are
deterministic).
"""

from __future__ import annotations

import pytest
import torch
import torch.nn as nn

import flash_mhc  # noqa: F401
from flash_mhc import MHCLiteBlock

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]


def _hot_path(inp):
    ops = torch.ops.flash_mhc
    x = inp["x"]
    T, n, C = x.shape
    xf = x.reshape(T, n * C)
    proj, inv = ops.fused_rmsnorm_project(xf, inp["W"])
    li = ops.fused_pre_map(x, inp["hp"])
    out = ops.fused_post_res(x, inp["lo"], inp["H"], inp["hq"])
    g4 = ops.fused_post_res_backward(inp["g4"], x, inp["lo"], inp["H"], inp["hq"])
    g3 = ops.fused_pre_map_backward(inp["g3"], x, inp["hp"])
    g1 = ops.fused_rmsnorm_project_backward(inp["gp"], xf, inp["W"], proj, inv)
    return [proj, inv, li, out, *g4, *g3, *g1]


def test_op_level_hot_path_graph_replay_matches_eager():
    torch.manual_seed(0)
    T, C = 8192, 1024
    d = "cuda"
    inp = {"x": torch.randn(T, 4, C, device=d).bfloat16(),
           "W": (torch.randn(32, 4 * C, device=d) * 0.02).bfloat16(),
           "lo": torch.randn(T, C, device=d).bfloat16(), "hp": torch.randn(T, 4, device=d),
           "hq": torch.randn(T, 4, device=d), "H": torch.randn(T, 4, 4, device=d),
           "g4": torch.randn(T, 4, C, device=d).bfloat16(), "g3": torch.randn(T, C, device=d).bfloat16(),
           "gp": torch.randn(T, 32, device=d).bfloat16()}
    eager = _hot_path(inp)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            _hot_path(inp)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        static = _hot_path(inp)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for a, b in zip(static, eager):
        assert torch.equal(a, b)


def test_block_fwd_bwd_graphed_matches_eager():
    """Whole-step capture: MHCLiteBlock forward + backward in one CUDA graph."""
    torch.manual_seed(1)
    T, C = 2048, 512
    layer = nn.Linear(C, C, bias=False)
    blk = MHCLiteBlock(4, C, layer).cuda().bfloat16().train()
    x = torch.randn(T, 4, C, device="cuda").bfloat16().requires_grad_(True)
    up = torch.randn(T, 4, C, device="cuda").bfloat16()

    def step():
        # The loss is formed inside the captured region (an upstream gradient
        # made on the default stream before capture would make autograd sync
        # with the legacy stream, which capture forbids for any op).
        out = blk(x)
        (out * up).sum().backward()
        return out

    out = step()
    ref = [out.detach().clone(), x.grad.clone()] + [p.grad.clone() for p in blk.parameters()]
    # Drop the eager graph: its nodes would keep the leaves' gradient
    # accumulators created on the default stream, which a capture cannot use.
    del out
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            blk.zero_grad(set_to_none=True)
            x.grad = None
            step()
    torch.cuda.current_stream().wait_stream(s)
    blk.zero_grad(set_to_none=True)
    x.grad = None
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        static_out = step()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    got = [static_out.detach(), x.grad] + [p.grad for p in blk.parameters()]
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
