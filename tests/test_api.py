"""Drop-in API checks (CPU): op schemas, fakes, module layout, CPU block path."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import flash_mhc
from flash_mhc import MHCLiteBlock, build_permutation_matrices
from flash_mhc import ops as fops
from tests._util import GOLDEN, assert_close, load_golden

API = json.loads((GOLDEN / "reference_api.json").read_text())

REF_OPS = [
    "fused_rmsnorm_project", "fused_rmsnorm_project_bwd_dx", "fused_pre_map",
    "fused_pre_map_backward", "fused_post_res", "fused_post_res_backward",
]


@pytest.mark.parametrize("name", REF_OPS)
def test_schema_identical_to_reference(name):
    op = getattr(torch.ops.flash_mhc, name).default
    assert str(op._schema) == API["schemas"][name]


def test_fake_impls_match_reference_shapes_and_dtypes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    T, n, C = 8, 4, 16
    with FakeTensorMode():
        x = torch.empty(T, n, C, dtype=torch.bfloat16)
        xf = torch.empty(T, n * C, dtype=torch.bfloat16)
        W = torch.empty(32, n * C, dtype=torch.bfloat16)
        h = torch.empty(T, n, dtype=torch.float32)
        H = torch.empty(T, n, n, dtype=torch.float32)
        lo = torch.empty(T, C, dtype=torch.bfloat16)
        go1 = torch.empty(T, 32, dtype=torch.bfloat16)
        rows = {
            "fused_rmsnorm_project": torch.ops.flash_mhc.fused_rmsnorm_project(xf, W),
            "fused_rmsnorm_project_bwd_dx": torch.ops.flash_mhc.fused_rmsnorm_project_bwd_dx(
                go1, xf, W, go1, h[:, 0].contiguous()),
            "fused_pre_map": torch.ops.flash_mhc.fused_pre_map(x, h),
            "fused_pre_map_backward": torch.ops.flash_mhc.fused_pre_map_backward(lo, x, h),
            "fused_post_res": torch.ops.flash_mhc.fused_post_res(x, lo, H, h),
            "fused_post_res_backward": torch.ops.flash_mhc.fused_post_res_backward(x, x, lo, H, h),
        }
        for k, v in rows.items():
            vs = v if isinstance(v, tuple) else (v,)
            got = [[list(t.shape), str(t.dtype)] for t in vs]
            assert got == API["fake"][k], k
        gx, gW = torch.ops.flash_mhc.fused_rmsnorm_project_backward(go1, xf, W, go1, h[:, 0])
        assert gx.shape == xf.shape and gW.shape == W.shape and gW.dtype == torch.bfloat16


def test_fake_impls_of_added_ops():
    """The ops this build adds (K2, the fused pre-block forward and the pieces
    of the block backward) have fake implementations with the CUDA impls'
    output shapes and dtypes, so they trace under torch.compile."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    ops = torch.ops.flash_mhc
    T, n, C = 8, 4, 16
    shp = lambda ts: [(tuple(t.shape), t.dtype) for t in (ts if isinstance(ts, tuple) else (ts,))]  # noqa: E731
    bf, f32 = torch.bfloat16, torch.float32
    with FakeTensorMode():
        x = torch.empty(T, n, C, dtype=bf)
        W = torch.empty(32, n * C, dtype=bf)
        proj = torch.empty(T, 32, dtype=bf)
        h = torch.empty(T, n, dtype=f32)
        H = torch.empty(T, n, n, dtype=f32)
        lo = torch.empty(T, C, dtype=bf)
        a = torch.empty(1, dtype=bf)
        bias = torch.empty(32, dtype=bf)
        perm = torch.empty(24, 16, dtype=f32)
        assert shp(ops.mhc_pre_forward(x, W, a, a, a, bias, perm)) == [
            ((T, C), bf), ((T, 32), bf), ((T,), f32), ((T, 4), f32), ((T, 4), f32),
            ((T, 4, 4), f32)]
        assert shp(ops.mhc_coeffs(proj, a, a, a, bias, perm)) == [
            ((T, 4), f32), ((T, 4), f32), ((T, 4, 4), f32)]
        assert shp(ops.mhc_coeffs_backward_split(h, h, H, proj, a, a, a, bias, perm)) == [
            ((T, 32), bf), ((1,), bf), ((1,), bf), ((1,), bf), ((32,), bf)]
        assert shp(ops.mhc_coeffs_backward(h, h, H, proj, a, a, a, bias, perm)) == [
            ((T, 32), bf), ((35,), f32)]
        assert shp(ops.pre_map_grad_h(lo, x, h)) == [((T, n), f32)]
        assert shp(ops.post_res_grad_params(x, x, lo, H, h)) == [
            ((T, C), bf), ((T, n, n), f32), ((T, n), f32)]
        assert shp(ops.mhc_grad_x_combine(x, lo, h, None)) == [((T, n, C), bf)]
        assert shp(ops.mhc_grad_x_combine_post(x, lo, h, x, H)) == [((T, n, C), bf)]


def test_ops_raise_on_cpu_tensors_like_reference():
    """No CPU kernel is registered (reference behaviour): CPU tensors raise."""
    x = torch.zeros(4, 4, 8, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        torch.ops.flash_mhc.fused_pre_map(x, torch.zeros(4, 4))


def test_state_dict_layout_identical_to_reference():
    blk = MHCLiteBlock(4, 16, nn.Linear(16, 16, bias=False))
    sd = {k: list(v.shape) for k, v in blk.state_dict().items()}
    assert sd == API["state_dict"]


def test_build_permutation_matrices_identical():
    m, idx = build_permutation_matrices(4)
    assert idx == API["perm4_identity_idx"]
    assert torch.equal(m, torch.tensor(API["perm4"]))
    m3, _ = build_permutation_matrices(3)
    assert m3.shape == (6, 9)


def test_exports_and_autotune_shim():
    assert set(flash_mhc.__all__) == {"MHCLiteBlock", "build_permutation_matrices"}
    with fops.disable_autotune_temporarily():
        assert fops._autotune_disable_depth() == 1
        with fops.disable_autotune_temporarily():
            assert fops._autotune_disable_depth() == 2
    assert fops._autotune_disable_depth() == 0


def test_path_predicate():
    blk = MHCLiteBlock(4, 8, nn.Identity())
    assert not blk._uses_fused_path(torch.zeros(2, 4, 8, dtype=torch.bfloat16))  # CPU
    blk3 = MHCLiteBlock(3, 8, nn.Identity())
    assert not blk3._uses_fused_path(torch.zeros(2, 3, 8))


class _IdentityLinear(nn.Module):
    """The reference test's stand-in layer: gelu(Linear(bias=False))."""

    def __init__(self, dim):
        super().__init__()
        self.proj = nn.Linear(dim, dim, bias=False)

    def forward(self, x, **kwargs):
        return F.gelu(self.proj(x))


def _block_from_golden(g, dtype, ckpt=False):
    C = int(g["C"])
    blk = MHCLiteBlock(4, C, _IdentityLinear(C), activation_checkpointing=ckpt)
    with torch.no_grad():
        blk.alpha_pre.copy_(torch.from_numpy(np.asarray(g["alpha_pre"])))
        blk.alpha_post.copy_(torch.from_numpy(np.asarray(g["alpha_post"])))
        blk.alpha_res.copy_(torch.from_numpy(np.asarray(g["alpha_res"])))
        blk.W_all.weight.copy_(torch.from_numpy(g["W"]))
        blk.W_all.bias.copy_(torch.from_numpy(g["bias"]))
        blk.layer.proj.weight.copy_(torch.from_numpy(g["Wl"]))
    return blk.to(dtype).train()


@pytest.mark.parametrize("ckpt", [False, True])
@pytest.mark.parametrize("name", ["block_fp32", "block_outlier_fp32"])
def test_cpu_block_reproduces_reference_golden(name, ckpt):
    """On CPU the block takes the pure-PyTorch path; it must reproduce the
    reference's own outputs and gradients on the same parameters and inputs."""
    g = load_golden(name)
    blk = _block_from_golden(g, torch.float32, ckpt)
    x = torch.from_numpy(g["x"]).requires_grad_(True)
    out = blk(x)
    (out * torch.from_numpy(g["g"])).sum().backward()
    assert_close("out", out.detach().numpy(), g["out"], 1e-6, 1e-5)
    assert_close("grad_x", x.grad.numpy(), g["grad_x"], 1e-6, 1e-5)
    for p, k in ((blk.W_all.weight, "g_W"), (blk.W_all.bias, "g_bias"),
                 (blk.alpha_pre, "g_alpha_pre"), (blk.alpha_post, "g_alpha_post"),
                 (blk.alpha_res, "g_alpha_res"), (blk.layer.proj.weight, "g_Wl")):
        scale = max(1.0, float(np.abs(g[k]).max()))
        assert_close(k, p.grad.numpy(), g[k], 1e-5 * scale, 1e-5)


def test_cpu_block_bf16_reproduces_reference_golden():
    g = load_golden("block_bf16")
    blk = _block_from_golden(g, torch.bfloat16)
    x = torch.from_numpy(g["x"]).to(torch.bfloat16).requires_grad_(True)
    out = blk(x)
    (out.float() * torch.from_numpy(g["g"])).sum().backward()
    # Same torch ops in the same order as the reference: bit-identical.
    assert_close("out", out.detach().float().numpy(), g["out"], 0, 0)
    assert_close("grad_x", x.grad.float().numpy(), g["grad_x"], 0, 0)
