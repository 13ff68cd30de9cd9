"""GPU parity of the six kernels (+ the K1 weight gradient) against the CPU oracle.

Every call goes through ``torch.ops.flash_mhc`` -> ctypes -> the C ABI of
libflashmhc_sm100.so.  Inputs are seeded; the oracle (oracle/mhc_oracle.py,
pinned to the reference in tests/test_oracle.py) computes in float64 on the
same bf16 inputs.

Tolerances (north star of this build):
* bf16 outputs: |got - ref| <= 2e-2 + 1e-2 * |ref|;
* f32 reductions (grad_h, grad_H, grad_h_post): |got - ref| <= 1e-4 * sum|terms|
  (the scale of f32 accumulation error; terms cancel, so |ref| is not a bound);
* inv_rms: relative 1e-5.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import flash_mhc  # noqa: F401  (registers torch.ops.flash_mhc)
from oracle import mhc_oracle as O
from tests._util import assert_close, assert_sum_close, load_golden

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]

BF_ATOL, BF_RTOL = 2e-2, 1e-2
RED_REL = 1e-4


def _bf(a, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(torch.bfloat16)


def _f32(a, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def _np(t):
    return t.detach().float().cpu().numpy()


def _inputs(T, C, seed, outlier=False):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, 4, C)).astype(np.float32)
    if outlier:
        cols = rng.choice(C, size=max(1, C // 100), replace=False)
        x[:, :, cols] *= 100.0
    x = O.bf16_round(x)
    lo = O.bf16_round(rng.standard_normal((T, C)))
    W = O.bf16_round(rng.standard_normal((32, 4 * C)) * 0.02)
    hp = rng.standard_normal((T, 4)).astype(np.float32)
    hpost = rng.standard_normal((T, 4)).astype(np.float32)
    H = rng.standard_normal((T, 4, 4)).astype(np.float32)
    g_pre = O.bf16_round(rng.standard_normal((T, C)))
    g_post = O.bf16_round(rng.standard_normal((T, 4, C)))
    g_proj = O.bf16_round(rng.standard_normal((T, 32)))
    return dict(x=x, lo=lo, W=W, hp=hp, hpost=hpost, H=H, g_pre=g_pre, g_post=g_post,
                g_proj=g_proj)


SHAPES = [
    (2048, 256, False),   # the reference test size (tests/test_correctness.py:95, 163, 206)
    (1, 64, False),       # tiny T
    (16, 768, True),      # edge config C=768 with 1% x100 outlier channels
    (257, 1024, False),   # T not a multiple of any tile
    (40, 100, False),     # C % 8 != 0 -> 4-wide vector path
    (33, 97, False),      # odd C -> scalar path
]


@pytest.mark.parametrize("T,C,outlier", SHAPES)
def test_k3_fwd_bwd(T, C, outlier):
    d = _inputs(T, C, 10 + T + C, outlier)
    x, hp, go = _bf(d["x"]), _f32(d["hp"]), _bf(d["g_pre"])
    out = torch.ops.flash_mhc.fused_pre_map(x, hp)
    assert out.dtype == torch.bfloat16 and out.shape == (T, C)
    assert_close("k3_fwd", _np(out), O.k3_fwd(d["x"], d["hp"]), BF_ATOL, BF_RTOL)
    gx, gh = torch.ops.flash_mhc.fused_pre_map_backward(go, x, hp)
    rgx, rgh = O.k3_bwd(d["g_pre"], d["x"], d["hp"])
    assert_close("k3_gx", _np(gx), rgx, BF_ATOL, BF_RTOL)
    assert gh.dtype == torch.float32
    assert_sum_close("k3_gh", _np(gh), rgh, O.k3_bwd_abs(d["g_pre"], d["x"]), RED_REL)


@pytest.mark.parametrize("T,C,outlier", SHAPES)
def test_k4_fwd_bwd(T, C, outlier):
    d = _inputs(T, C, 20 + T + C, outlier)
    x, lo, H, hpost, go = _bf(d["x"]), _bf(d["lo"]), _f32(d["H"]), _f32(d["hpost"]), _bf(d["g_post"])
    out = torch.ops.flash_mhc.fused_post_res(x, lo, H, hpost)
    assert out.shape == (T, 4, C)
    assert_close("k4_fwd", _np(out), O.k4_fwd(d["x"], d["lo"], d["H"], d["hpost"]), BF_ATOL,
                 BF_RTOL)
    gx, glo, gH, ghp = torch.ops.flash_mhc.fused_post_res_backward(go, x, lo, H, hpost)
    rgx, rglo, rgH, rghp = O.k4_bwd(d["g_post"], d["x"], d["lo"], d["H"], d["hpost"])
    sH, sP = O.k4_bwd_abs(d["g_post"], d["x"], d["lo"])
    assert_close("k4_gx", _np(gx), rgx, BF_ATOL, BF_RTOL)
    assert_close("k4_glo", _np(glo), rglo, BF_ATOL, BF_RTOL)
    assert_sum_close("k4_gH", _np(gH), rgH, sH, RED_REL)
    assert_sum_close("k4_ghp", _np(ghp), rghp, sP, RED_REL)


def _check_gw(got, go, xf, inv):
    ref = O.k1_bwd_dw(go, xf, inv)
    gos = O.bf16_round(go.astype(np.float64) * inv.astype(np.float64)[:, None]).astype(np.float64)
    scale = np.abs(gos).T @ np.abs(xf.astype(np.float64))
    diff = np.abs(got.astype(np.float64) - ref)
    lim = BF_RTOL * np.abs(ref) + RED_REL * scale + 1e-6
    assert np.all(diff <= lim), f"k1_gW: worst {np.max(diff / lim):.3g} x bound"


@pytest.mark.parametrize("T,C,outlier", SHAPES)
def test_k1_fwd_bwd(T, C, outlier):
    d = _inputs(T, C, 30 + T + C, outlier)
    xf_np = d["x"].reshape(T, 4 * C)
    xf, W, go = _bf(xf_np), _bf(d["W"]), _bf(d["g_proj"])
    out, inv = torch.ops.flash_mhc.fused_rmsnorm_project(xf, W)
    rout, rinv = O.k1_fwd(xf_np, d["W"])
    assert out.dtype == torch.bfloat16 and inv.dtype == torch.float32
    assert_close("k1_inv_rms", _np(inv), rinv, 0, 1e-5)
    assert_close("k1_out", _np(out), rout, BF_ATOL, BF_RTOL)
    # backward from the kernel's own proj/inv_rms (what autograd feeds it)
    proj_np, inv_np = _np(out), _np(inv)
    gx = torch.ops.flash_mhc.fused_rmsnorm_project_bwd_dx(go, xf, W, out, inv)
    rgx = O.k1_bwd_dx(d["g_proj"], xf_np, d["W"], proj_np, inv_np)
    assert_close("k1_gx", _np(gx), rgx, BF_ATOL, BF_RTOL)
    gx2, gW = torch.ops.flash_mhc.fused_rmsnorm_project_backward(go, xf, W, out, inv)
    assert torch.equal(gx, gx2)
    _check_gw(_np(gW), d["g_proj"], xf_np, inv_np)


def test_k1_autograd_contract():
    """fused_rmsnorm_project's registered autograd returns (grad_x, grad_W)."""
    d = _inputs(64, 64, 5)
    xf_np = d["x"].reshape(64, 256)
    xf = _bf(xf_np).requires_grad_(True)
    W = _bf(d["W"]).requires_grad_(True)
    out, inv = torch.ops.flash_mhc.fused_rmsnorm_project(xf, W)
    go = _bf(d["g_proj"])
    (out.float() * go.float()).sum().backward()
    rgx = O.k1_bwd_dx(d["g_proj"], xf_np, d["W"], _np(out), _np(inv))
    assert_close("grad_x", _np(xf.grad), rgx, BF_ATOL, BF_RTOL)
    _check_gw(_np(W.grad), d["g_proj"], xf_np, _np(inv))


def test_golden_inputs_through_cuda_ops():
    """The reference-generated fixture inputs, through the CUDA ops, against the
    oracle (tight) and against the reference restatements (the reference
    test's own tolerances, tests/test_correctness.py:48-51)."""
    g = load_golden("ops_bf16")
    T = int(g["T"])
    out, inv = torch.ops.flash_mhc.fused_rmsnorm_project(_bf(g["k1_x"]), _bf(g["k1_W"]))
    assert_close("k1 vs oracle", _np(out), O.k1_fwd(g["k1_x"], g["k1_W"])[0], BF_ATOL, BF_RTOL)
    assert_close("k1 vs reference", _np(out), g["k1_out"], 1e-2, 1.6e-2)
    out = torch.ops.flash_mhc.fused_pre_map(_bf(g["k3_x"]), _f32(g["k3_h"]))
    assert_close("k3 vs reference", _np(out), g["k3_out"], 1e-2, 1.6e-2)
    gx, gh = torch.ops.flash_mhc.fused_pre_map_backward(_bf(g["k3_go"]), _bf(g["k3_x"]),
                                                        _f32(g["k3_h"]))
    assert_close("k3 gx vs reference", _np(gx), g["k3_gx"], 5e-2, 2e-2)
    assert_close("k3 gh vs reference", _np(gh), g["k3_gh"], 5e-2, 2e-2)
    out = torch.ops.flash_mhc.fused_post_res(_bf(g["k4_x"]), _bf(g["k4_lo"]), _f32(g["k4_H"]),
                                             _f32(g["k4_hp"]))
    assert_close("k4 vs reference", _np(out), g["k4_out"], 1e-2, 1.6e-2)
    r = torch.ops.flash_mhc.fused_post_res_backward(_bf(g["k4_go"]), _bf(g["k4_x"]),
                                                    _bf(g["k4_lo"]), _f32(g["k4_H"]),
                                                    _f32(g["k4_hp"]))
    for got, k in zip(r, ("k4_gx", "k4_glo", "k4_gH", "k4_ghp")):
        assert_close(k + " vs reference", _np(got), g[k], 5e-2, 2e-2)
    assert T == 64


def test_zero_tokens():
    x = torch.empty(0, 4, 64, device="cuda", dtype=torch.bfloat16)
    assert torch.ops.flash_mhc.fused_pre_map(x, torch.empty(0, 4, device="cuda")).shape == (0, 64)
    out, inv = torch.ops.flash_mhc.fused_rmsnorm_project(
        x.reshape(0, 256), torch.zeros(32, 256, device="cuda", dtype=torch.bfloat16))
    assert out.shape == (0, 32) and inv.shape == (0,)


def test_non_contiguous_inputs_are_handled():
    """The reference assumes contiguity silently; here inputs are made contiguous."""
    d = _inputs(64, 128, 3)
    x = _bf(d["x"])
    xt = x.transpose(0, 1).contiguous().transpose(0, 1)  # same values, non-contiguous
    assert not xt.is_contiguous()
    hp = _f32(d["hp"])
    assert torch.equal(torch.ops.flash_mhc.fused_pre_map(xt, hp),
                       torch.ops.flash_mhc.fused_pre_map(x, hp))


def test_n_not_4_raises_value_error():
    x = torch.zeros(8, 3, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        torch.ops.flash_mhc.fused_pre_map(x, torch.zeros(8, 3, device="cuda"))


def test_full_size_against_torch_fp32():
    """Metric shape T=65536, C=1024: the kernels against a torch float32
    restatement on the GPU (the CPU oracle would take minutes at this size)."""
    torch.manual_seed(0)
    T, C = 65536, 1024
    x = torch.randn(T, 4, C, device="cuda").bfloat16()
    lo = torch.randn(T, C, device="cuda").bfloat16()
    H = torch.randn(T, 4, 4, device="cuda")
    hp = torch.randn(T, 4, device="cuda")
    go = torch.randn(T, 4, C, device="cuda").bfloat16()
    xf32, lof, gof = x.float(), lo.float(), go.float()
    out = torch.ops.flash_mhc.fused_post_res(x, lo, H, hp)
    ref = torch.einsum("tij,tjc->tic", H, xf32) + hp[:, :, None] * lof[:, None, :]
    torch.testing.assert_close(out.float(), ref, atol=BF_ATOL, rtol=BF_RTOL)
    del out, ref
    gx, glo, gH, ghp = torch.ops.flash_mhc.fused_post_res_backward(go, x, lo, H, hp)
    torch.testing.assert_close(glo.float(), torch.einsum("ti,tic->tc", hp, gof), atol=BF_ATOL,
                               rtol=BF_RTOL)
    torch.testing.assert_close(gx.float(), torch.einsum("tij,tic->tjc", H, gof), atol=BF_ATOL,
                               rtol=BF_RTOL)
    sH = torch.einsum("tic,tjc->tij", gof.abs(), xf32.abs())
    dH = (gH - torch.einsum("tic,tjc->tij", gof, xf32)).abs()
    assert bool((dH <= RED_REL * sH).all())
    dP = (ghp - torch.einsum("tic,tc->ti", gof, lof)).abs()
    assert bool((dP <= RED_REL * torch.einsum("tic,tc->ti", gof.abs(), lof.abs())).all())
    del gx, glo, gH, ghp
    h = torch.randn(T, 4, device="cuda")
    out = torch.ops.flash_mhc.fused_pre_map(x, h)
    torch.testing.assert_close(out.float(), torch.einsum("tj,tjc->tc", h, xf32), atol=BF_ATOL,
                               rtol=BF_RTOL)
    W = (torch.randn(32, 4 * C, device="cuda") * 0.02).bfloat16()
    xf = x.reshape(T, 4 * C)
    proj, inv = torch.ops.flash_mhc.fused_rmsnorm_project(xf, W)
    rinv = torch.rsqrt((xf.float() ** 2).mean(1) + 1e-6)
    torch.testing.assert_close(inv, rinv, atol=0, rtol=1e-5)
    rproj = (xf.float() @ W.float().t()) * rinv[:, None]
    torch.testing.assert_close(proj.float(), rproj, atol=BF_ATOL, rtol=BF_RTOL)


def _kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}


@pytest.mark.parametrize("T,kernel", [(1, "k1_fwd_rows_cluster_kernel"),
                                      (148, "k1_fwd_rows_cluster_kernel"),
                                      (150, "k1_fwd_rows_kernel"),
                                      (4096, "k1_fwd_tc_splitk_kernel")])
def test_small_t_k1_forward_kernel_choice(T, kernel):
    """Few tokens: clusters of CTAs per token pair while the pairs are too few to
    fill the GPU, then one block per pair, then the split-K tensor-core kernel."""
    xf = torch.randn(T, 3072, device="cuda").bfloat16()
    W = (torch.randn(32, 3072, device="cuda") * 0.02).bfloat16()
    names = _kernel_names(lambda: torch.ops.flash_mhc.fused_rmsnorm_project(xf, W))
    assert any(kernel in n and (kernel != "k1_fwd_rows_kernel" or "cluster" not in n)
               for n in names), names


def test_metric_shape_runs_the_tensor_core_k1():
    """At T=65536, nC=4096 the K1 forward and backward are the TMA + tcgen05 kernels."""
    d = _inputs(256, 1024, 9)
    xf = torch.randn(65536, 4096, device="cuda").bfloat16()
    W = _bf(np.tile(d["W"], (1, 1)))
    names = _kernel_names(lambda: torch.ops.flash_mhc.fused_rmsnorm_project(xf, W))
    assert any("k1_fwd_tc_kernel" in n for n in names), names
    out, inv = torch.ops.flash_mhc.fused_rmsnorm_project(xf, W)
    go = torch.randn(65536, 32, device="cuda").bfloat16()
    names = _kernel_names(
        lambda: torch.ops.flash_mhc.fused_rmsnorm_project_backward(go, xf, W, out, inv))
    assert any("k1_bwd_tc_kernel" in n for n in names), names


@pytest.mark.parametrize("T,C", [(1, 256), (31, 256), (33, 256), (60, 256), (148, 256),
                                 (150, 256), (1000, 256), (4733, 256),
                                 (3000, 1024), (129, 2048),
                                 (65536, 64),   # 2 k-chunks: 74 CTAs add into each
                                 (20000, 1024),  # groups of 4 k-chunks, 18 or 19 CTAs each
                                 (6000, 768)])  # groups of 2, 12 or 13 CTAs each, nC = 3072
def test_k1_token_partitioning(T, C):
    """Forward: token pairs split over clusters of 8, 4 and 2 CTAs (T = 1 .. 148),
    one block per pair (150), token ranges split across CTAs in 32-row units,
    partial tiles.
    Backward: the k-chunks form groups of G (1, 2, 4 or 8, chosen per shape),
    each CTA of a group takes every ng-th token tile; groups of unequal CTA
    counts, fewer tiles than CTAs, partial token tiles; grad_W reduction."""
    d = _inputs(T, C, 40 + T)
    xf_np = d["x"].reshape(T, 4 * C)
    xf, W, go = _bf(xf_np), _bf(d["W"]), _bf(d["g_proj"])
    out, inv = torch.ops.flash_mhc.fused_rmsnorm_project(xf, W)
    rout, rinv = O.k1_fwd(xf_np, d["W"])
    assert_close("inv_rms", _np(inv), rinv, 0, 1e-5)
    assert_close("out", _np(out), rout, BF_ATOL, BF_RTOL)
    gx, gW = torch.ops.flash_mhc.fused_rmsnorm_project_backward(go, xf, W, out, inv)
    rgx = O.k1_bwd_dx(d["g_proj"], xf_np, d["W"], _np(out), _np(inv))
    assert_close("gx", _np(gx), rgx, BF_ATOL, BF_RTOL)
    _check_gw(_np(gW), d["g_proj"], xf_np, _np(inv))
    gx_only = torch.ops.flash_mhc.fused_rmsnorm_project_bwd_dx(go, xf, W, out, inv)
    assert torch.equal(gx_only, gx)
    # deterministic: a second call gives identical bits
    gx2, gW2 = torch.ops.flash_mhc.fused_rmsnorm_project_backward(go, xf, W, out, inv)
    assert torch.equal(gx2, gx) and torch.equal(gW2, gW)


def test_no_device_error_recorded():
    """No bounded wait of the tensor-core kernels expired during this module."""
    from flash_mhc import _native

    assert _native.check_device_error() == 0


def test_k1_tensor_core_kernels_are_bitwise_deterministic_at_metric_shape():
    """Repeated runs at T=65536, nC=4096 give identical bits (fixed reduction
    orders, no atomics); a race between pipeline roles would show up here."""
    torch.manual_seed(3)
    xf = torch.randn(65536, 4096, device="cuda").bfloat16()
    W = (torch.randn(32, 4096, device="cuda") * 0.02).bfloat16()
    go = torch.randn(65536, 32, device="cuda").bfloat16()
    out0, inv0 = torch.ops.flash_mhc.fused_rmsnorm_project(xf, W)
    gx0, gW0 = torch.ops.flash_mhc.fused_rmsnorm_project_backward(go, xf, W, out0, inv0)
    for _ in range(8):
        out, inv = torch.ops.flash_mhc.fused_rmsnorm_project(xf, W)
        gx, gW = torch.ops.flash_mhc.fused_rmsnorm_project_backward(go, xf, W, out0, inv0)
        assert torch.equal(out, out0) and torch.equal(inv, inv0)
        assert torch.equal(gx, gx0) and torch.equal(gW, gW0)
    rinv = torch.rsqrt((xf.float() ** 2).mean(1) + 1e-6)
    torch.testing.assert_close(inv0, rinv, atol=0, rtol=1e-5)
    s = (go.float() * out0.float()).sum(1) * inv0 * inv0 / 4096
    rgx = inv0[:, None] * (go.float() @ W.float()) - s[:, None] * xf.float()
    torch.testing.assert_close(gx0.float(), rgx, atol=BF_ATOL, rtol=BF_RTOL)
    gos = (go.float() * inv0[:, None]).bfloat16().float()
    rgW = gos.t() @ xf.float()
    torch.testing.assert_close(gW0.float(), rgW, atol=BF_ATOL, rtol=BF_RTOL)


@pytest.mark.parametrize("T,C", [(300, 768), (40, 100), (33, 97)])
def test_block_backward_pieces(T, C):
    """pre_map_grad_h (K3 backward without grad_x) and the one-pass grad_x
    combination used by the fused block backward."""
    d = _inputs(T, C, 60 + T)
    x, hp, gli = _bf(d["x"]), _f32(d["hp"]), _bf(d["g_pre"])
    gx_ref, gh_ref = torch.ops.flash_mhc.fused_pre_map_backward(gli, x, hp)
    gh = torch.ops.flash_mhc.pre_map_grad_h(gli, x, hp)
    assert torch.equal(gh, gh_ref)
    g = torch.Generator(device="cuda").manual_seed(T)
    gx1 = torch.randn(T, 4, C, device="cuda", generator=g).bfloat16()
    gx4 = torch.randn(T, 4, C, device="cuda", generator=g).bfloat16()
    for extra in (gx4, None):
        out = torch.ops.flash_mhc.mhc_grad_x_combine(gx1, gli, hp, extra)
        ref = gx1.float() + hp[:, :, None] * gli.float()[:, None, :]
        if extra is not None:
            ref = ref + extra.float()
        torch.testing.assert_close(out.float(), ref, atol=BF_ATOL, rtol=BF_RTOL)

    # K4 backward without grad_x gives the other three gradients bit for bit,
    # and the combination forms K4's grad_x term from g_out and H itself.
    lo, H, hpost, g_out = _bf(d["lo"]), _f32(d["H"]), _f32(d["hpost"]), _bf(d["g_post"])
    k4_ref = torch.ops.flash_mhc.fused_post_res_backward(g_out, x, lo, H, hpost)
    k4 = torch.ops.flash_mhc.post_res_grad_params(g_out, x, lo, H, hpost)
    for got, want in zip(k4, k4_ref[1:]):
        assert torch.equal(got, want)
    out = torch.ops.flash_mhc.mhc_grad_x_combine_post(gx1, gli, hp, g_out, H)
    ref = (gx1.float() + hp[:, :, None] * gli.float()[:, None, :]
           + torch.einsum("tij,tic->tjc", H, g_out.float()))
    torch.testing.assert_close(out.float(), ref, atol=BF_ATOL, rtol=BF_RTOL)


def test_large_token_sharded_config_rows():
    """The large per-GPU config (131,072 tokens x C = 4096: every (T, 4, C)
    tensor has more than 2^31 elements).  All six ops run on the full tensors;
    a sample of rows, first and last included, is checked against a float32
    restatement, so 64-bit offsets and the last partial tiles are exercised."""
    T, C = 131072, 4096
    ops = torch.ops.flash_mhc
    g = torch.Generator(device="cuda").manual_seed(11)
    rn = lambda *s, std=1.0: (torch.randn(*s, device="cuda", generator=g) * std)  # noqa: E731
    x = rn(T, 4, C).bfloat16()
    W = rn(32, 4 * C, std=0.02).bfloat16()
    lo = rn(T, C).bfloat16()
    hp, hq, H = rn(T, 4), rn(T, 4), rn(T, 4, 4)
    gp, g3, g4 = rn(T, 32).bfloat16(), rn(T, C).bfloat16(), rn(T, 4, C).bfloat16()
    xf = x.view(T, 4 * C)
    proj, inv = ops.fused_rmsnorm_project(xf, W)
    li = ops.fused_pre_map(x, hp)
    out = ops.fused_post_res(x, lo, H, hq)
    gx4, glo, gH, ghp = ops.fused_post_res_backward(g4, x, lo, H, hq)
    gx3, gh3 = ops.fused_pre_map_backward(g3, x, hp)
    gx1, gW = ops.fused_rmsnorm_project_backward(gp, xf, W, proj, inv)
    rows = torch.cat([torch.arange(0, 64), torch.randint(64, T - 64, (192,), generator=torch.Generator().manual_seed(5)),
                      torch.arange(T - 64, T)]).cuda()
    f = lambda t: t[rows].float()  # noqa: E731
    xr, xfr, lor, g4r, g3r = f(x), f(xf), f(lo), f(g4), f(g3)
    rinv = torch.rsqrt((xfr ** 2).mean(1) + 1e-6)
    torch.testing.assert_close(inv[rows], rinv, atol=0, rtol=1e-5)
    torch.testing.assert_close(f(proj), (xfr @ W.float().t()) * rinv[:, None], atol=BF_ATOL, rtol=BF_RTOL)
    torch.testing.assert_close(f(li), (hp[rows][:, :, None] * xr).sum(1), atol=BF_ATOL, rtol=BF_RTOL)
    Hr, hqr = H[rows], hq[rows]
    torch.testing.assert_close(f(out), torch.einsum("tij,tjc->tic", Hr, xr) + hqr[:, :, None] * lor[:, None, :],
                               atol=BF_ATOL, rtol=BF_RTOL)
    torch.testing.assert_close(f(gx4), torch.einsum("tij,tic->tjc", Hr, g4r), atol=BF_ATOL, rtol=BF_RTOL)
    torch.testing.assert_close(f(glo), (hqr[:, :, None] * g4r).sum(1), atol=BF_ATOL, rtol=BF_RTOL)
    torch.testing.assert_close(gH[rows], torch.einsum("tic,tjc->tij", g4r, xr), atol=1e-1, rtol=1e-3)
    torch.testing.assert_close(gx3[rows].float(), hp[rows][:, :, None] * g3r[:, None, :], atol=BF_ATOL, rtol=BF_RTOL)
    torch.testing.assert_close(gh3[rows], (xr * g3r[:, None, :]).sum(2), atol=1e-1, rtol=1e-3)
    s = (f(gp) * f(proj)).sum(1) * inv[rows] ** 2 / (4 * C)
    rgx1 = inv[rows][:, None] * (f(gp) @ W.float()) - s[:, None] * xfr
    torch.testing.assert_close(f(gx1), rgx1, atol=BF_ATOL, rtol=BF_RTOL)
    assert torch.isfinite(gW.float()).all()
