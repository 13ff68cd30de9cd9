"""GPU parity of ``MHCLiteBlock`` (fused CUDA path) against the reference.

* the reference's own pure-PyTorch bf16 path, captured in tests/golden/block_bf16.npz
  (reference end-to-end tolerances, tests/test_correctness.py:284, 296, 317);
* the reference's float32 pure-PyTorch block on bf16-valued seeded inputs
  (tests/golden/block_cfg0_fp32.npz at BASELINE configs[0], block_grid_fp32.npz),
  at the stated bounds: bf16 outputs within 2e-2 + 1e-2*|ref|, coefficients
  within 1e-4, parameter gradients within 2e-2*max|ref| + 1e-2*|ref|;
* the float64 oracle block (oracle.mhc_oracle.block_forward_backward) run with
  K1's eps;
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
    # bf16 outputs within 2e-2 + 1e-2 |ref| (the coefficients are f32)
    assert_close("out", out.detach().float().cpu().numpy(), r["out"], 2e-2, 1e-2)
    assert_close("grad_x", x.grad.float().cpu().numpy(), r["grad_x"], 2e-2, 1e-2)


class _GridLayer(nn.Module):
    """The wrapped layer of the bf16-grid fixtures: proj(x), or gelu(proj(x))."""

    def __init__(self, C, gelu):
        super().__init__()
        self.proj = nn.Linear(C, C, bias=False)
        self.gelu = gelu

    def forward(self, x, **kwargs):
        y = self.proj(x)
        return F.gelu(y) if self.gelu else y


@pytest.mark.parametrize("name", ["block_cfg0_fp32", "block_grid_fp32"])
def test_block_matches_reference_fp32_at_north_star_bounds(name):
    """The fused bf16 block against the reference's float32 pure-PyTorch block
    (src/flash_mhc/block.py:126-148) on the same values: every input and
    parameter is a bf16 value (tests/golden/block_inputs.py), so the only
    differences are this path's own roundings (bf16 logits, layer input,
    layer output of the bf16 layer, block output, and in the backward the
    bf16 gradients it stores).

    Bounds, with no term that depends on the data's conditioning:
    * block output and grad_x (bf16 outputs): |d| <= 2e-2 + 1e-2 |ref|;
    * h_pre, h_post, H_merged (f32 coefficients, configs[0] init): |d| <= 1e-4;
    * parameter gradients (sums over all T tokens, bf16 for a bf16 module):
      |d| <= 2e-2 max|ref| + 1e-2 |ref| per tensor (for an alpha, a scalar,
      3% of |ref|).
    configs[0] is BASELINE's CPU reference config (T=4096, C=1024, default
    init, Linear(1024, 1024)); the grid case moves the alphas to 0.7-1.3 and
    wraps a gelu layer.
    """
    from tests.golden.block_inputs import block_case_inputs

    g = load_golden(name)
    T, C = int(g["T"]), int(g["C"])
    inp = block_case_inputs(T, C, int(g["seed"]), float(g["wl_std"]), tuple(g["alphas"]))
    layer = _GridLayer(C, bool(int(g["gelu"])))
    blk = MHCLiteBlock(4, C, layer)
    with torch.no_grad():
        for p, v in zip((blk.alpha_pre, blk.alpha_post, blk.alpha_res), inp["alphas"]):
            p.fill_(float(v))
        blk.W_all.weight.copy_(torch.from_numpy(inp["W"]))
        blk.W_all.bias.copy_(torch.from_numpy(inp["bias"]))
        layer.proj.weight.copy_(torch.from_numpy(inp["Wl"]))
    blk = blk.cuda().to(torch.bfloat16).train()
    x = torch.from_numpy(inp["x"]).cuda().to(torch.bfloat16).requires_grad_(True)
    assert blk._uses_fused_path(x)
    out = blk(x)
    out.backward(torch.from_numpy(inp["g"]).cuda().to(torch.bfloat16))
    rows = torch.from_numpy(g["rows"]).cuda()
    assert_close("out", out.detach()[rows].float().cpu().numpy(), g["out"], 2e-2, 1e-2)
    assert_close("grad_x", x.grad[rows].float().cpu().numpy(), g["grad_x"], 2e-2, 1e-2)
    if name == "block_cfg0_fp32":
        with torch.no_grad():
            _li, _p, _i, h_pre, h_post, H = torch.ops.flash_mhc.mhc_pre_forward(
                x.detach(), blk.W_all.weight, blk.alpha_pre, blk.alpha_post, blk.alpha_res,
                blk.W_all.bias, blk.perm_mat)
        for k, t in (("h_pre", h_pre), ("h_post", h_post), ("H_merged", H)):
            assert_close(k, t[rows].cpu().numpy(), g[k], 1e-4, 0.0)
    grads = _grads(blk)
    grads["g_Wl_rows"] = layer.proj.weight.grad[torch.from_numpy(g["wl_rows"]).cuda()]
    del grads["g_Wl"]
    for k, t in grads.items():
        ref = g[k]
        assert_close(k, t.float().cpu().numpy().reshape(ref.shape), ref,
                     2e-2 * float(np.abs(ref).max()), 1e-2)


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
    # The reference's bf16 path rounds every op of K2 to bf16 (about eight
    # roundings on the way to H_merged) while the fused K2 keeps f32, so the
    # coefficients may differ by a few bf16 steps (2^-8 each near 1), which the
    # post-mix multiplies by |x| (x100 in the outlier channels) and by
    # |layer_output|: bound = 5e-2 + 2e-2|ref| + 2^-6 (sum_j |x_j| + |lo|).
    with torch.no_grad():
        lo = blk.layer(blk._mhc_pre_map_pytorch(xb)[0]).float()
    cond = xb.float().abs().sum(dim=1, keepdim=True) + lo.abs()[:, None, :]
    lim = 5e-2 + 2e-2 * ref.float().abs() + 2.0 ** -6 * cond
    diff = (ref.float() - out.float()).abs()
    assert bool((diff <= lim).all()), float((diff / lim).max())
    params = dict(alpha_pre=0.01, alpha_post=0.01, alpha_res=0.01,
                  W=blk.W_all.weight.detach().float().cpu().numpy(),
                  bias=blk.W_all.bias.detach().float().cpu().numpy(),
                  perm=blk.perm_mat.float().cpu().numpy(),
                  Wl=blk.layer.weight.detach().float().cpu().numpy())
    xn = xb.float().cpu().numpy()
    r = O.block_forward_backward(params, xn, np.zeros((T, 4, C)), rms_eps=1e-6, layer="linear")
    # With x100 outlier channels the layer input and output reach ~100s, and
    # their bf16 rounding (the bf16 layer input, the bf16 layer) and that of
    # the bf16 logits K2 reads scale with |x| and |lo|.
    # Bound: 5e-2 + 2e-2*|ref| + 2^-7 * (sum_j |x_j| + |lo|).
    got = out.float().cpu().numpy()
    cond = np.abs(xn).sum(axis=1, keepdims=True) + np.abs(r["layer_input"] @ params["Wl"].T)[:, None, :]
    lim = 5e-2 + 2e-2 * np.abs(r["out"]) + 2.0 ** -7 * cond
    diff = np.abs(got - r["out"])
    assert np.all(diff <= lim), f"out vs oracle: worst {np.max(diff / lim):.3g} x bound"
