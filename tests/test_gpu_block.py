"""GPU parity of ``MHCLiteBlock`` (fused CUDA path) against the reference.

* the reference's own pure-PyTorch bf16 path, captured in tests/golden/block_bf16.npz
  (reference end-to-end tolerances, tests/test_correctness.py:284, 296, 317);
* the float64 oracle block (oracle.mhc_oracle.block_forward_backward) run with
  K1's eps, bf16 outputs within 2e-2 + 1e-2*|ref|;
* the pure-PyTorch path of the same module on the same GPU at larger shapes,
  including T=65537 (tail) and eval/no-grad tiny T with outlier channels.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from flash_mhc import MHCLiteBlock
from oracle import mhc_oracle as O
from tests._util import assert_close, load_golden

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]


class _IdentityLinear(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.proj = nn.Linear(dim, dim, bias=False)

    def forward(self, x, **kwargs):
        return F.gelu(self.proj(x))


def _golden_block(g):
    C = int(g["C"])
    blk = MHCLiteBlock(4, C, _IdentityLinear(C))
    with torch.no_grad():
        blk.alpha_pre.copy_(torch.from_numpy(np.asarray(g["alpha_pre"])))
        blk.alpha_post.copy_(torch.from_numpy(np.asarray(g["alpha_post"])))
        blk.alpha_res.copy_(torch.from_numpy(np.asarray(g["alpha_res"])))
        blk.W_all.weight.copy_(torch.from_numpy(g["W"]))
        blk.W_all.bias.copy_(torch.from_numpy(g["bias"]))
        blk.layer.proj.weight.copy_(torch.from_numpy(g["Wl"]))
    return blk.cuda().to(torch.bfloat16).train()


def _grads(blk):
    return {
        "g_W": blk.W_all.weight.grad, "g_bias": blk.W_all.bias.grad,
        "g_alpha_pre": blk.alpha_pre.grad, "g_alpha_post": blk.alpha_post.grad,
        "g_alpha_res": blk.alpha_res.grad, "g_Wl": blk.layer.proj.weight.grad,
    }


def test_block_matches_reference_golden():
    g = load_golden("block_bf16")
    blk = _golden_block(g)
    x = torch.from_numpy(g["x"]).cuda().to(torch.bfloat16).requires_grad_(True)
    assert blk._uses_fused_path(x)
    out = blk(x)
    (out.float() * torch.from_numpy(g["g"]).cuda()).sum().backward()
    assert_close("E2E_fwd", out.detach().float().cpu().numpy(), g["out"], 5e-2, 2e-2)
    assert_close("E2E_grad_x", x.grad.float().cpu().numpy(), g["grad_x"], 1e-1, 5e-2)
    for k, t in _grads(blk).items():
        ref = g[k]
        scale = max(1.0, float(np.abs(ref).max()))
        assert_close(k, t.float().cpu().numpy().reshape(ref.shape), ref, 1e-1 * scale, 5e-2)


def test_block_matches_float64_oracle():
    """The fused path against the float64 restatement using K1's eps (1e-6)."""
    g = load_golden("block_bf16")
    blk = _golden_block(g)
    x = torch.from_numpy(g["x"]).cuda().to(torch.bfloat16).requires_grad_(True)
    out = blk(x)
    (out.float() * torch.from_numpy(g["g"]).cuda()).sum().backward()
    params = dict(alpha_pre=float(blk.alpha_pre.detach().float()),
                  alpha_post=float(blk.alpha_post.detach().float()),
                  alpha_res=float(blk.alpha_res.detach().float()),
                  W=blk.W_all.weight.detach().float().cpu().numpy(),
                  bias=blk.W_all.bias.detach().float().cpu().numpy(), perm=g["perm"],
                  Wl=blk.layer.proj.weight.detach().float().cpu().numpy())
    r = O.block_forward_backward(params, g["x"], g["g"], rms_eps=1e-6)
    # h_pre, h_post and H_merged are rounded to bf16 (as in the reference), an
    # error of up to 2^-8 of their magnitude that the output multiplies by |x|
    # and |layer_output|: bound = 2e-2 + 1e-2|ref| + 2^-8 (sum_j |x_j| + |lo|).
    got = out.detach().float().cpu().numpy()
    cond = np.abs(g["x"]).sum(axis=1, keepdims=True) + np.abs(
        O.gelu(r["layer_input"] @ params["Wl"].T))[:, None, :]
    lim = 2e-2 + 1e-2 * np.abs(r["out"]) + 2.0 ** -8 * cond
    diff = np.abs(got - r["out"])
    assert np.all(diff <= lim), f"out vs oracle: worst {np.max(diff / lim):.3g} x bound"
    assert_close("grad_x", x.grad.float().cpu().numpy(), r["grad_x"], 1e-1, 5e-2)


def _make(T, C, seed, layer="linear"):
    torch.manual_seed(seed)
    lay = nn.Linear(C, C, bias=False)
    with torch.no_grad():
        lay.weight.normal_(0.0, 0.02)
    blk = MHCLiteBlock(4, C, lay).cuda().to(torch.bfloat16)
    return blk


def _run(blk, x, g, fused):
    blk.zero_grad(set_to_none=True)
    xx = x.detach().clone().requires_grad_(True)
    out = blk._forward_triton(xx) if fused else blk._forward_pytorch(xx)
    (out.float() * g.float()).sum().backward()
    return out.detach(), xx.grad, {n: p.grad.clone() for n, p in blk.named_parameters()}


@pytest.mark.parametrize("T,C", [(4096, 1024), (65537, 768), (65536, 2048)])  # last: the block config
def test_fused_vs_pytorch_path_same_gpu(T, C):
    blk = _make(T, C, 1).train()
    torch.manual_seed(2)
    x = torch.randn(T, 4, C, device="cuda").bfloat16()
    g = torch.randn(T, 4, C, device="cuda").bfloat16()
    o1, gx1, p1 = _run(blk, x, g, True)
    o2, gx2, p2 = _run(blk, x, g, False)
    torch.testing.assert_close(o1.float(), o2.float(), atol=5e-2, rtol=2e-2)
    torch.testing.assert_close(gx1.float(), gx2.float(), atol=1e-1, rtol=5e-2)
    for k in p2:
        scale = max(1.0, float(p2[k].float().abs().max()))
        torch.testing.assert_close(p1[k].float(), p2[k].float(), atol=1e-1 * scale, rtol=5e-2)


def test_activation_checkpointing_is_bitwise_neutral():
    T, C = 2048, 512
    blk = _make(T, C, 3).train()
    torch.manual_seed(4)
    x = torch.randn(T, 4, C, device="cuda").bfloat16()
    g = torch.randn(T, 4, C, device="cuda").bfloat16()
    blk.activation_checkpointing = False
    o1, gx1, p1 = _run(blk, x, g, True)
    blk.activation_checkpointing = True
    o2, gx2, p2 = _run(blk, x, g, True)
    assert torch.equal(o1, o2) and torch.equal(gx1, gx2)
    for k in p1:
        assert torch.equal(p1[k], p2[k]), k


@pytest.mark.parametrize("T", [1, 16, 256])
def test_eval_no_grad_tiny_T_with_outliers(T):
    C = 768
    blk = _make(T, C, 5).eval()
    rng = np.random.default_rng(T)
    x = rng.standard_normal((T, 4, C)).astype(np.float32)
    x[:, :, rng.choice(C, size=C // 100, replace=False)] *= 100.0
    xb = torch.from_numpy(x).cuda().to(torch.bfloat16)
    with torch.no_grad():
        out = blk(xb)  # the no-grad fast path (no autograd Functions, no op dispatch)
        ref = blk._forward_pytorch(xb)
    assert out.shape == (T, 4, C)
    # Same kernels as the grad-enabled path, so the same bits.
    assert torch.equal(blk(xb).detach(), out)
    # Both paths round the coefficients to bf16 but at different points (the
    # fused K2 keeps f32 intermediates), so they may differ by one bf16 step of
    # a coefficient, multiplied by |x| (x100 in the outlier channels) and by
    # |layer_output|: bound = 5e-2 + 2e-2|ref| + 2^-7 (sum_j |x_j| + |lo|).
    with torch.no_grad():
        lo = blk.layer(blk._mhc_pre_map_pytorch(xb)[0]).float()
    cond = xb.float().abs().sum(dim=1, keepdim=True) + lo.abs()[:, None, :]
    lim = 5e-2 + 2e-2 * ref.float().abs() + 2.0 ** -7 * cond
    diff = (ref.float() - out.float()).abs()
    assert bool((diff <= lim).all()), float((diff / lim).max())
    params = dict(alpha_pre=0.01, alpha_post=0.01, alpha_res=0.01,
                  W=blk.W_all.weight.detach().float().cpu().numpy(),
                  bias=blk.W_all.bias.detach().float().cpu().numpy(),
                  perm=blk.perm_mat.float().cpu().numpy(),
                  Wl=blk.layer.weight.detach().float().cpu().numpy())
    xn = xb.float().cpu().numpy()
    r = O.block_forward_backward(params, xn, np.zeros((T, 4, C)), rms_eps=1e-6, layer="linear")
    # K2 runs in bf16 (as in the reference), so H_merged and h_post carry an
    # absolute error of ~2^-8; with x100 outlier channels that error is
    # multiplied by |x|.  Bound: 5e-2 + 2e-2*|ref| + 2^-7 * (sum_j |x_j| + |lo|).
    got = out.float().cpu().numpy()
    cond = np.abs(xn).sum(axis=1, keepdims=True) + np.abs(r["layer_input"] @ params["Wl"].T)[:, None, :]
    lim = 5e-2 + 2e-2 * np.abs(r["out"]) + 2.0 ** -7 * cond
    diff = np.abs(got - r["out"])
    assert np.all(diff <= lim), f"out vs oracle: worst {np.max(diff / lim):.3g} x bound"
