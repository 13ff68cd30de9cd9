"""GPU parity of flash_mhc::mhc_pre_forward (C ABI fmhc_mhc_pre_fwd): K1 with
K2 in its epilogue, then K3 -- at T <= 888 all three in one kernel.

* every output equals the separate ops fused_rmsnorm_project -> mhc_coeffs ->
  fused_pre_map bit for bit, on each K1 kernel's range: the small-T row kernel
  (with and without K3 inside), the split-K cluster kernel (S = 4 and 2), the
  persistent tensor-core kernel (with a tail tile) and the CUDA-core kernel;
  parameters in f32 and in bf16;
* the layer input and coefficients against the float64 oracle
  (oracle.mhc_oracle.k1_fwd / k2_coeffs / k3_fwd) on a small case.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import flash_mhc  # noqa: F401
from flash_mhc import build_permutation_matrices
from oracle import mhc_oracle as O
from tests._util import assert_close

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]


def _inputs(T, C, pdtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, 4, C, device="cuda", generator=g).bfloat16()
    W = (torch.randn(32, 4 * C, device="cuda", generator=g) * 0.02).bfloat16()
    a = [torch.full((1,), v, device="cuda", dtype=pdtype) for v in (0.7, 0.9, 1.3)]
    bias = (torch.randn(32, device="cuda", generator=g) * 0.5).to(pdtype)
    perm = build_permutation_matrices(4)[0].to(device="cuda", dtype=pdtype)
    return x, W, a, bias, perm


# (T, C): the small-T kernels -- token pairs over clusters of 8, 4 or 2 CTAs
# (T <= 148) and one block per pair -- with K3 inside (C % 8 == 0) and with K3
# separate (C = 20, 36), split-K S = 4 (T = 889, 4096) and S = 2 (8192), the
# persistent tensor-core kernel (20000; 65537 with a tail tile), the CUDA-core
# kernel (nC = 80 is no multiple of the tensor-core k-step).
SHAPES = [(1, 768), (2, 768), (3, 1024), (16, 768), (60, 768), (148, 64), (149, 768),
          (256, 768), (888, 1024), (5, 20), (300, 36), (889, 1024), (4096, 1024), (8192, 768),
          (20000, 768), (65537, 1024), (1000, 20)]


@pytest.mark.parametrize("pdtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("T,C", SHAPES)
def test_pre_forward_equals_separate_ops(T, C, pdtype):
    ops = torch.ops.flash_mhc
    x, W, (a_pre, a_post, a_res), bias, perm = _inputs(T, C, pdtype, seed=T + C)
    with torch.no_grad():
        li, proj, inv, hp, hq, H = ops.mhc_pre_forward(x, W, a_pre, a_post, a_res, bias, perm)
        proj2, inv2 = ops.fused_rmsnorm_project(x.reshape(T, 4 * C), W)
        hp2, hq2, H2 = ops.mhc_coeffs(proj2, a_pre, a_post, a_res, bias, perm)
        li2 = ops.fused_pre_map(x, hp2)
    for name, a, b in (("proj", proj, proj2), ("inv_rms", inv, inv2), ("h_pre", hp, hp2),
                       ("h_post", hq, hq2), ("H_merged", H, H2), ("layer_input", li, li2)):
        assert a.shape == b.shape and a.dtype == b.dtype, name
        assert torch.equal(a, b), f"{name}: max |diff| {(a.float() - b.float()).abs().max().item()}"


@pytest.mark.parametrize("T,C", [(7, 64), (1500, 256)])
def test_pre_forward_matches_float64_oracle(T, C):
    x, W, (a_pre, a_post, a_res), bias, perm = _inputs(T, C, torch.float32, seed=3)
    with torch.no_grad():
        li, proj, inv, hp, hq, H = torch.ops.flash_mhc.mhc_pre_forward(
            x, W, a_pre, a_post, a_res, bias, perm)
    xf = x.float().cpu().numpy()
    r_proj, r_inv = O.k1_fwd(xf.reshape(T, 4 * C), W.float().cpu().numpy())
    assert_close("proj", proj.float().cpu().numpy(), r_proj, 2e-2, 1e-2)
    assert_close("inv_rms", inv.cpu().numpy(), r_inv, 1e-4, 1e-4)
    # K2 and K3 from the kernel's own proj, so only their arithmetic is compared
    ap, aq, ar = (float(O.bf16_round(np.float32(v)).reshape(-1)[0]) for v in (0.7, 0.9, 1.3))
    ctx = O.k2_coeffs(proj.float().cpu().numpy(), ap, aq, ar,
                      O.bf16_round(bias.float().cpu().numpy()), perm.float().cpu().numpy())
    assert_close("h_pre", hp.cpu().numpy(), ctx["h_pre"], 1e-2, 1e-2)
    assert_close("h_post", hq.cpu().numpy(), ctx["h_post"], 1e-2, 1e-2)
    assert_close("H_merged", H.cpu().numpy(), ctx["H_merged"], 2e-2, 2e-2)
    r_li = O.k3_fwd(xf, hp.cpu().numpy())
    assert_close("layer_input", li.float().cpu().numpy(), r_li, 2e-2, 1e-2)


def test_pre_forward_empty_batch():
    x, W, (a_pre, a_post, a_res), bias, perm = _inputs(0, 64, torch.float32, seed=1)
    outs = torch.ops.flash_mhc.mhc_pre_forward(x, W, a_pre, a_post, a_res, bias, perm)
    assert [tuple(o.shape) for o in outs] == [(0, 64), (0, 32), (0,), (0, 4), (0, 4), (0, 4, 4)]
