"""Pin the CPU oracle (oracle/mhc_oracle.py) against tensors made by the reference.

The fixtures under tests/golden/ were produced by tests/golden/make_golden.py,
which imports the reference package and its test-file restatements.  These
tests run on the CPU (no GPU, no CUDA library needed).
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from oracle import mhc_oracle as O
from tests._util import GOLDEN, assert_close, load_golden

# Reference tolerances (tests/test_correctness.py:48-51, 284, 296, 317).
FWD_ATOL, FWD_RTOL = 1e-2, 1.6e-2
BWD_ATOL, BWD_RTOL = 5e-2, 2e-2


def test_bf16_round_matches_torch():
    rng = np.random.default_rng(0)
    v = np.concatenate([
        rng.standard_normal(100000).astype(np.float32) * 10.0 ** rng.integers(-30, 30, 100000),
        np.array([0.0, -0.0, np.inf, -np.inf, 3.3895314e38, 1e-40, -1e-42, 65504.0], np.float32),
    ]).astype(np.float32)
    ours = O.bf16_round(v)
    theirs = torch.from_numpy(v).to(torch.bfloat16).float().numpy()
    assert np.array_equal(ours.view(np.uint32), theirs.view(np.uint32))
    # NaN stays NaN
    assert np.isnan(O.bf16_round(np.array([np.nan], np.float32)))[0]


def test_permutation_matrices_match_reference():
    api = json.loads((GOLDEN / "reference_api.json").read_text())
    mats, idx = O.build_permutation_matrices(4)
    assert idx == api["perm4_identity_idx"] == 0
    assert np.array_equal(mats, np.array(api["perm4"], np.float32))
    assert np.array_equal(mats[0].reshape(4, 4), np.eye(4))
    # every row is a permutation matrix, all distinct
    m = mats.reshape(24, 4, 4)
    assert np.all(m.sum(1) == 1) and np.all(m.sum(2) == 1)
    assert len({r.tobytes() for r in mats}) == 24


def test_ops_fp32_match_reference_restatements():
    g = load_golden("ops_fp32")
    out, inv = O.k1_fwd(g["k1_x"], g["k1_W"], bf16=False)
    assert_close("k1_out", out, g["k1_out"], 1e-6, 1e-5)
    assert_close("k1_inv_rms", inv, g["k1_inv_rms"], 0, 1e-6)
    gx = O.k1_bwd_dx(g["k1_go"], g["k1_x"], g["k1_W"], out, inv, bf16=False)
    assert_close("k1_gx", gx, g["k1_gx"], 1e-6, 1e-5)
    gW = O.k1_bwd_dw(g["k1_go"], g["k1_x"], inv, bf16=False)
    assert_close("k1_gW", gW, g["k1_gW"], 1e-5, 1e-5)

    out = O.k3_fwd(g["k3_x"], g["k3_h"], bf16=False)
    assert_close("k3_out", out, g["k3_out"], 1e-6, 1e-5)
    gx, gh = O.k3_bwd(g["k3_go"], g["k3_x"], g["k3_h"], bf16=False)
    assert_close("k3_gx", gx, g["k3_gx"], 1e-6, 1e-5)
    assert_close("k3_gh", gh, g["k3_gh"], 1e-5, 1e-5)

    out = O.k4_fwd(g["k4_x"], g["k4_lo"], g["k4_H"], g["k4_hp"], bf16=False)
    assert_close("k4_out", out, g["k4_out"], 1e-6, 1e-5)
    gx, glo, gH, ghp = O.k4_bwd(g["k4_go"], g["k4_x"], g["k4_lo"], g["k4_H"], g["k4_hp"], bf16=False)
    assert_close("k4_gx", gx, g["k4_gx"], 1e-5, 1e-5)
    assert_close("k4_glo", glo, g["k4_glo"], 1e-5, 1e-5)
    assert_close("k4_gH", gH, g["k4_gH"], 1e-5, 1e-5)
    assert_close("k4_ghp", ghp, g["k4_ghp"], 1e-5, 1e-5)


def test_ops_bf16_match_reference_restatements():
    """bf16 restatements round at different points (e.g. the K1 test reference
    rounds the raw projection to bf16 before scaling), so the comparison uses
    the reference test's own bf16 tolerances."""
    g = load_golden("ops_bf16")
    out, inv = O.k1_fwd(g["k1_x"], g["k1_W"])
    assert_close("k1_out", out, g["k1_out"], FWD_ATOL, FWD_RTOL)
    assert_close("k1_inv_rms", inv, g["k1_inv_rms"], 0, 1e-5)
    gx = O.k1_bwd_dx(g["k1_go"], g["k1_x"], g["k1_W"], out, inv)
    assert_close("k1_gx", gx, g["k1_gx"], BWD_ATOL, BWD_RTOL)
    gW = O.k1_bwd_dw(g["k1_go"], g["k1_x"], inv)
    assert_close("k1_gW", gW, g["k1_gW"], BWD_ATOL, BWD_RTOL)

    out = O.k3_fwd(g["k3_x"], g["k3_h"])
    assert_close("k3_out", out, g["k3_out"], FWD_ATOL, FWD_RTOL)
    gx, gh = O.k3_bwd(g["k3_go"], g["k3_x"], g["k3_h"])
    assert_close("k3_gx", gx, g["k3_gx"], BWD_ATOL, BWD_RTOL)
    assert_close("k3_gh", gh, g["k3_gh"], BWD_ATOL, BWD_RTOL)

    out = O.k4_fwd(g["k4_x"], g["k4_lo"], g["k4_H"], g["k4_hp"])
    assert_close("k4_out", out, g["k4_out"], FWD_ATOL, FWD_RTOL)
    gx, glo, gH, ghp = O.k4_bwd(g["k4_go"], g["k4_x"], g["k4_lo"], g["k4_H"], g["k4_hp"])
    assert_close("k4_gx", gx, g["k4_gx"], BWD_ATOL, BWD_RTOL)
    assert_close("k4_glo", glo, g["k4_glo"], BWD_ATOL, BWD_RTOL)
    assert_close("k4_gH", gH, g["k4_gH"], BWD_ATOL, BWD_RTOL)
    assert_close("k4_ghp", ghp, g["k4_ghp"], BWD_ATOL, BWD_RTOL)


def _block_params(g):
    return dict(alpha_pre=g["alpha_pre"][0], alpha_post=g["alpha_post"][0],
                alpha_res=g["alpha_res"][0], W=g["W"], bias=g["bias"], perm=g["perm"], Wl=g["Wl"])


@pytest.mark.parametrize("name", ["block_fp32", "block_outlier_fp32"])
def test_block_fp32_matches_reference(name):
    """The float64 block restatement (forward AND hand-derived backward) against
    the reference's pure-PyTorch path run in float32."""
    g = load_golden(name)
    r = O.block_forward_backward(_block_params(g), g["x"], g["g"], rms_eps=float(g["rms_eps"]))
    assert_close("out", r["out"], g["out"], 1e-5, 1e-4)
    assert_close("h_pre", r["h_pre"], g["h_pre"], 1e-6, 1e-4)
    assert_close("h_post", r["h_post"], g["h_post"], 1e-6, 1e-4)
    assert_close("H_merged", r["H_merged"], g["H_merged"], 1e-6, 1e-4)
    assert_close("layer_input", r["layer_input"], g["layer_input"], 1e-5, 1e-4)
    assert_close("grad_x", r["grad_x"], g["grad_x"], 1e-5, 1e-4)
    gr = r["grads"]
    for k, gk in (("alpha_pre", "g_alpha_pre"), ("alpha_post", "g_alpha_post"),
                  ("alpha_res", "g_alpha_res"), ("W", "g_W"), ("bias", "g_bias"), ("Wl", "g_Wl")):
        ref = g[gk]
        scale = max(1.0, float(np.abs(ref).max()))
        assert_close(gk, np.reshape(gr[k], ref.shape), ref, 1e-4 * scale, 1e-4)


@pytest.mark.parametrize("name", ["block_grid_fp32", "block_cfg0_fp32"])
def test_block_grid_fixtures_match_oracle(name):
    """The bf16-grid fixtures (the reference's float32 block on bf16-valued
    seeded inputs, tests/golden/block_inputs.py) against the float64 block
    restatement: forward, coefficients and every gradient to f32 accuracy."""
    from tests.golden.block_inputs import block_case_inputs

    g = load_golden(name)
    T, C, seed = int(g["T"]), int(g["C"]), int(g["seed"])
    inp = block_case_inputs(T, C, seed, float(g["wl_std"]), tuple(g["alphas"]))
    params = dict(alpha_pre=inp["alphas"][0], alpha_post=inp["alphas"][1],
                  alpha_res=inp["alphas"][2], W=inp["W"], bias=inp["bias"],
                  perm=O.build_permutation_matrices(4)[0], Wl=inp["Wl"])
    layer = "linear_gelu" if int(g["gelu"]) else "linear"
    r = O.block_forward_backward(params, inp["x"], inp["g"], rms_eps=float(np.finfo(np.float32).eps),
                                 layer=layer)
    rows = g["rows"]
    for k in ("out", "grad_x", "h_pre", "h_post", "H_merged", "layer_input"):
        assert_close(k, r[k][rows], g[k], 1e-5, 1e-4)
    gr = r["grads"]
    for k, gk in (("alpha_pre", "g_alpha_pre"), ("alpha_post", "g_alpha_post"),
                  ("alpha_res", "g_alpha_res"), ("W", "g_W"), ("bias", "g_bias")):
        ref = g[gk]
        assert_close(gk, np.reshape(gr[k], ref.shape), ref, 1e-4 * max(1.0, float(np.abs(ref).max())), 1e-4)
    ref = g["g_Wl_rows"]
    assert_close("g_Wl", gr["Wl"][g["wl_rows"]], ref, 1e-4 * max(1.0, float(np.abs(ref).max())), 1e-4)


def test_block_bf16_matches_reference_within_bf16_tolerance():
    """The reference's bf16 path rounds every intermediate; the oracle computes
    in float64 from the same bf16 inputs.  The reference's own end-to-end
    tolerances apply (tests/test_correctness.py:284, 296, 317)."""
    g = load_golden("block_bf16")
    r = O.block_forward_backward(_block_params(g), g["x"], g["g"], rms_eps=float(g["rms_eps"]))
    assert_close("out", r["out"], g["out"], 5e-2, 2e-2)
    assert_close("grad_x", r["grad_x"], g["grad_x"], 1e-1, 5e-2)
    gr = r["grads"]
    for k, gk in (("alpha_pre", "g_alpha_pre"), ("alpha_post", "g_alpha_post"),
                  ("alpha_res", "g_alpha_res"), ("W", "g_W"), ("bias", "g_bias"), ("Wl", "g_Wl")):
        ref = g[gk]
        scale = max(1.0, float(np.abs(ref).max()))
        assert_close(gk, np.reshape(gr[k], ref.shape), ref, 1e-1 * scale, 5e-2)


def test_oracle_self_consistency_k1_grad_matches_block_formula():
    """K1's fused backward (project, then scale) equals the chain rule through
    normalise-then-project when both are evaluated in float64."""
    rng = np.random.default_rng(7)
    T, nC, D = 16, 128, 32
    x = rng.standard_normal((T, nC))
    W = rng.standard_normal((D, nC)) * 0.02
    go = rng.standard_normal((T, D))
    out, inv = O.k1_fwd(x, W, bf16=False)
    gx = O.k1_bwd_dx(go, x, W, out, inv, bf16=False)
    eps = 1e-6
    # finite differences on a few coordinates
    for t, k in ((0, 0), (3, 17), (15, 127)):
        def f(xx):
            r = 1.0 / np.sqrt((xx[t] ** 2).mean() + eps)
            return float(((xx[t] @ W.T) * r) @ go[t])
        h = 1e-6
        xp, xm = x.copy(), x.copy()
        xp[t, k] += h
        xm[t, k] -= h
        fd = (f(xp) - f(xm)) / (2 * h)
        assert abs(fd - gx[t, k]) <= 1e-4 * max(1.0, abs(fd))


def test_fast_f32_step_agrees_with_float64_step():
    """The float32 step timed as the CPU baseline computes the same results."""
    rng = np.random.default_rng(11)
    T, C = 24, 64
    x = O.bf16_round(rng.standard_normal((T, 4, C)))
    W = O.bf16_round(rng.standard_normal((32, 4 * C)) * 0.02)
    lo = O.bf16_round(rng.standard_normal((T, C)))
    H = rng.standard_normal((T, 4, 4)).astype(np.float32)
    hq = rng.standard_normal((T, 4)).astype(np.float32)
    hp = rng.standard_normal((T, 4)).astype(np.float32)
    gp = O.bf16_round(rng.standard_normal((T, 32)))
    g3 = O.bf16_round(rng.standard_normal((T, C)))
    g4 = O.bf16_round(rng.standard_normal((T, 4, C)))
    a = O.hot_path_step(x, W, lo, H, hq, hp, gp, g3, g4)
    b = O.hot_path_step_f32(x, W, lo, H, hq, hp, gp, g3, g4)
    flat_a = [a[0], a[1], a[2], a[3], *a[4], *a[5], a[6], a[7]]
    flat_b = [b[0], b[1], b[2], b[3], *b[4], *b[5], b[6], b[7]]
    for i, (u, v) in enumerate(zip(flat_a, flat_b)):
        assert_close(f"step[{i}]", v, u, 2e-2, 1e-2)
