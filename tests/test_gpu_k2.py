"""GPU parity of the fused K2 kernels (flash_mhc::mhc_coeffs and its backward).

* forward against the reference's eager K2 in bf16 (the block's own
  `_coeffs_from_proj`, i.e. src/flash_mhc/block.py:161-169, on the same GPU):
  the reference rounds every op to bf16, the kernel keeps f32, so they agree
  to a few bf16 steps; against the same code in float32 (parameters rounded
  to bf16 as the reference's ``.to(dt)``) within 1e-5;
* forward and backward against the float64 oracle (oracle.mhc_oracle.k2_coeffs
  and its hand-derived backward): f32 coefficients within 1e-5, bf16
  grad_proj within 2e-2 + 1e-2*|ref|, parameter gradients (f32 sums over T)
  within 1e-4 * sum_t |term|.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import flash_mhc  # noqa: F401
from flash_mhc import MHCLiteBlock
from oracle import mhc_oracle as O
from tests._util import assert_close, assert_sum_close

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]


def _setup(T, seed, alphas=(0.7, 0.9, 1.3), scale=1.0):
    torch.manual_seed(seed)
    blk = MHCLiteBlock(4, 16, torch.nn.Identity()).cuda()
    with torch.no_grad():
        blk.alpha_pre.fill_(alphas[0]); blk.alpha_post.fill_(alphas[1]); blk.alpha_res.fill_(alphas[2])
        blk.W_all.bias.normal_(0.0, 0.5)
    proj = (torch.randn(T, 32, device="cuda") * scale).bfloat16()
    return blk, proj


@pytest.mark.parametrize("T,scale", [(1, 1.0), (257, 1.0), (4096, 3.0), (65536, 1.0)])
def test_k2_forward_matches_reference_eager_bf16(T, scale):
    blk, proj = _setup(T, 1, scale=scale)
    h_pre, h_post, H = torch.ops.flash_mhc.mhc_coeffs(proj, blk.alpha_pre, blk.alpha_post,
                                                      blk.alpha_res, blk.W_all.bias, blk.perm_mat)
    with torch.no_grad():
        r_pre, r_post, r_H = blk._coeffs_from_proj(proj, torch.bfloat16)
    # The bf16 eager code rounds every op: H_merged = H_res - h_post h_pre
    # subtracts two bf16-rounded terms of magnitude up to 1 and 2 (half-steps
    # 2^-9 and 2^-8) computed from bf16-rounded sigmoids and softmax, so it is
    # off the f32 value by up to ~3e-2 absolute.
    torch.testing.assert_close(h_pre, r_pre.float(), atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(h_post, r_post.float(), atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(H, r_H.float(), atol=3e-2, rtol=2e-2)
    # f32 coefficients: the reference's K2 evaluated in float32 on the same
    # bf16 logits, with the parameters rounded to bf16 as its `.to(dt)` does
    with torch.no_grad():
        for p in (blk.alpha_pre, blk.alpha_post, blk.alpha_res, blk.W_all.bias):
            p.copy_(p.bfloat16().float())
        f_pre, f_post, f_H = blk._coeffs_from_proj(proj.float(), torch.float32)
    torch.testing.assert_close(h_pre, f_pre, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(h_post, f_post, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(H, f_H, atol=1e-5, rtol=1e-5)


def _oracle_params(blk):
    return dict(ap=blk.alpha_pre.item(), aq=blk.alpha_post.item(), ar=blk.alpha_res.item(),
                bias=O.bf16_round(blk.W_all.bias.detach().float().cpu().numpy()),
                perm=blk.perm_mat.float().cpu().numpy())


@pytest.mark.parametrize("T", [3, 1000])
def test_k2_forward_backward_match_float64_oracle(T):
    blk, proj = _setup(T, 2)
    p = _oracle_params(blk)
    ap, aq, ar = (float(O.bf16_round(np.float32(v)).reshape(-1)[0]) for v in (p["ap"], p["aq"], p["ar"]))
    pr = proj.float().cpu().numpy()
    ctx = O.k2_coeffs(pr, ap, aq, ar, p["bias"], p["perm"])
    with torch.no_grad():
        a, b, c = torch.ops.flash_mhc.mhc_coeffs(proj, blk.alpha_pre, blk.alpha_post,
                                                 blk.alpha_res, blk.W_all.bias, blk.perm_mat)
    # f32 coefficients from the same bf16 logits and bf16-rounded parameters
    assert_close("h_pre", a.cpu().numpy(), ctx["h_pre"], 1e-5, 1e-5)
    assert_close("h_post", b.cpu().numpy(), ctx["h_post"], 1e-5, 1e-5)
    assert_close("H_merged", c.cpu().numpy(), ctx["H_merged"], 1e-5, 1e-5)

    g = torch.Generator(device="cuda").manual_seed(5)
    g_hpre = torch.randn(T, 4, device="cuda", generator=g)
    g_hpost = torch.randn(T, 4, device="cuda", generator=g)
    g_H = torch.randn(T, 4, 4, device="cuda", generator=g)
    with torch.no_grad():
        g_proj, gp = torch.ops.flash_mhc.mhc_coeffs_backward(
            g_hpre, g_hpost, g_H, proj, blk.alpha_pre, blk.alpha_post, blk.alpha_res,
            blk.W_all.bias, blk.perm_mat)
    rg = O.k2_coeffs_bwd(ctx, g_hpre.cpu().numpy(), g_hpost.cpu().numpy(), g_H.cpu().numpy(),
                         ap, aq, ar, p["perm"])
    r_proj, r_ap, r_aq, r_ar, r_bias = rg
    # grad_proj is a bf16 output: 2e-2 + 1e-2 |ref|
    assert_close("grad_proj", g_proj.float().cpu().numpy(), r_proj, 2e-2, 1e-2)
    # The parameter gradients are f32 sums over tokens of per-token terms
    # (the logit gradients z times the logit, or z alone for the bias); their
    # rounding error is bounded by a multiple of sum_t |term|, not of |sum|.
    ref_params = np.concatenate([[r_ap, r_aq, r_ar], r_bias])
    ap_s, aq_s, ar_s = (float(v) for v in (ap, aq, ar))
    z = np.concatenate([r_proj[:, :4] / ap_s, r_proj[:, 4:8] / aq_s, r_proj[:, 8:] / ar_s], axis=1)
    terms_abs = np.concatenate([
        [np.abs(z[:, :4] * pr[:, :4]).sum(), np.abs(z[:, 4:8] * pr[:, 4:8]).sum(),
         np.abs(z[:, 8:] * pr[:, 8:]).sum()],
        np.abs(z).sum(axis=0)])
    assert_sum_close("param_grads", gp.cpu().numpy(), ref_params, terms_abs, 1e-4)


def test_k2_autograd_through_block_params():
    """d(loss)/d(params) of mhc_coeffs via autograd equals the backward op."""
    blk, proj = _setup(512, 3)
    proj = proj.requires_grad_(True)
    a, b, c = torch.ops.flash_mhc.mhc_coeffs(proj, blk.alpha_pre, blk.alpha_post, blk.alpha_res,
                                             blk.W_all.bias, blk.perm_mat)
    loss = (a * 1.5).sum() + (b * -0.5).sum() + (c * 2.0).sum()
    loss.backward()
    g_proj, gp = torch.ops.flash_mhc.mhc_coeffs_backward(
        torch.full_like(a, 1.5), torch.full_like(b, -0.5), torch.full_like(c, 2.0), proj.detach(),
        blk.alpha_pre, blk.alpha_post, blk.alpha_res, blk.W_all.bias, blk.perm_mat)
    assert torch.equal(proj.grad, g_proj)
    assert torch.equal(blk.W_all.bias.grad, gp[3:])
    assert torch.equal(blk.alpha_res.grad, gp[2:3])


@pytest.mark.parametrize("param_dtype", [torch.float32, torch.bfloat16])
def test_k2_typed_entry_matches_packed_entry(param_dtype):
    """fmhc_k2_fwd_typed (parameters read where they live, f32 or bf16) gives
    the same bits as fmhc_k2_fwd on the packed f32 copy of the parameters."""
    from flash_mhc import _native

    blk, proj = _setup(1000, 11)
    blk = blk.to(param_dtype)
    a = [blk.alpha_pre, blk.alpha_post, blk.alpha_res]
    packed = torch.cat([t.reshape(-1) for t in a] + [blk.W_all.bias.reshape(-1)]).float().contiguous()
    perm32 = blk.perm_mat.float().contiguous()
    T = proj.shape[0]
    outs = []
    for typed in (False, True):
        hp = torch.empty(T, 4, device="cuda")
        hq = torch.empty(T, 4, device="cuda")
        H = torch.empty(T, 4, 4, device="cuda")
        st = torch.cuda.current_stream().cuda_stream
        if typed:
            dt = 1 if param_dtype == torch.bfloat16 else 0
            _native.call("fmhc_k2_fwd_typed", proj.data_ptr(), a[0].data_ptr(), a[1].data_ptr(),
                         a[2].data_ptr(), blk.W_all.bias.data_ptr(), dt, blk.perm_mat.data_ptr(), dt,
                         hp.data_ptr(), hq.data_ptr(), H.data_ptr(), T, st)
        else:
            _native.call("fmhc_k2_fwd", proj.data_ptr(), packed.data_ptr(), perm32.data_ptr(),
                         hp.data_ptr(), hq.data_ptr(), H.data_ptr(), T, st)
        outs.append((hp, hq, H))
    for x, y in zip(*outs):
        assert torch.equal(x, y)
    # and the op (which takes the typed entry for f32/bf16 parameters)
    got = torch.ops.flash_mhc.mhc_coeffs(proj, *a, blk.W_all.bias, blk.perm_mat)
    for x, y in zip(got, outs[0]):
        assert torch.equal(x, y)


@pytest.mark.parametrize("param_dtype", [torch.float32, torch.bfloat16])
def test_k2_backward_split_matches_packed(param_dtype):
    """mhc_coeffs_backward_split (parameters read in place, one gradient per
    parameter written in its dtype) gives the packed op's values: the same f32
    sums, rounded once to the parameter dtype."""
    blk, proj = _setup(3000, 12)
    blk = blk.to(param_dtype)
    T = proj.shape[0]
    g = torch.Generator(device="cuda").manual_seed(5)
    ghp = torch.randn(T, 4, device="cuda", generator=g)
    ghq = torch.randn(T, 4, device="cuda", generator=g)
    gH = torch.randn(T, 4, 4, device="cuda", generator=g)
    args = (ghp, ghq, gH, proj, blk.alpha_pre, blk.alpha_post, blk.alpha_res, blk.W_all.bias,
            blk.perm_mat)
    gproj_ref, gp = torch.ops.flash_mhc.mhc_coeffs_backward(*args)
    gproj, ga, gb, gc, gbias = torch.ops.flash_mhc.mhc_coeffs_backward_split(*args)
    assert torch.equal(gproj, gproj_ref)
    for got, ref in ((ga, gp[0:1]), (gb, gp[1:2]), (gc, gp[2:3]), (gbias, gp[3:35])):
        assert got.dtype == param_dtype
        assert torch.equal(got.reshape(-1), ref.to(param_dtype))
