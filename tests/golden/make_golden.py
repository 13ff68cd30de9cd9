"""Generate the golden fixtures in this folder from the reference implementation.

Run once, in a container where the reference project is available:

    python tests/golden/make_golden.py --reference-root <path to flash-mHC checkout>

It imports the reference package (``src/flash_mhc``) and its test module
(``tests/test_correctness.py``) in THIS process, so it must not be run in a
process that already imported this repository's ``flash_mhc`` (both define the
``flash_mhc`` torch.library namespace).  Everything runs on the CPU with fixed
seeds.  Outputs (all small):

* ``ops_fp32.npz`` / ``ops_bf16.npz``: inputs, outputs and autograd gradients
  of the reference test-file restatements of K1, K3 and K4
  (tests/test_correctness.py:99-123, 165-169, 208-214) for a random upstream
  gradient.
* ``block_fp32.npz`` / ``block_bf16.npz`` / ``block_outlier_fp32.npz``:
  ``MHCLiteBlock._forward_pytorch`` (src/flash_mhc/block.py:126-148) forward,
  grad_x and every parameter gradient, plus the K2 intermediates.
* ``block_cfg0_fp32.npz`` / ``block_grid_fp32.npz``: the same float32 block
  on bf16-valued seeded inputs and parameters (``block_inputs.py``), at
  BASELINE configs[0] (T=4096, C=1024, default init, Linear(1024, 1024)) and
  at a small stress case; per-token outputs for a stored subset of rows.
* ``reference_api.json``: op schemas, fake-impl output dtypes, the block's
  state_dict names/shapes and ``build_permutation_matrices(4)``.

Bit patterns of bf16 tensors are stored as uint16 so the fixtures are exact.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _np(t: torch.Tensor):
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy().copy()


def _ops_case(tc, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    T, n, C = 64, 4, 64
    nC, D = n * C, 32
    out = {"T": T, "n": n, "C": C, "D": D}

    def rn(*shape, std=1.0, dt=dtype):
        return (torch.randn(*shape, generator=g) * std).to(dt)

    # K1 (tests/test_correctness.py:99-123) -- W ~ N(0, 0.02) as in the bench config
    x = rn(T, nC).requires_grad_(True)
    W = rn(D, nC, std=0.02).requires_grad_(True)
    ref, inv = tc.TestK1FusedRMSNormProject._ref_fwd(None, x, W)
    go = rn(T, D)
    (ref.float() * go.float()).sum().backward()
    out.update(k1_x=_np(x), k1_W=_np(W), k1_out=_np(ref), k1_inv_rms=_np(inv.float()),
               k1_go=_np(go), k1_gx=_np(x.grad), k1_gW=_np(W.grad))

    # K3 (tests/test_correctness.py:165-169)
    x = rn(T, n, C).requires_grad_(True)
    h = torch.randn(T, n, generator=g).requires_grad_(True)
    ref = tc.TestK3FusedPreMap._ref_fwd(None, x, h)
    go = rn(T, C)
    (ref.float() * go.float()).sum().backward()
    out.update(k3_x=_np(x), k3_h=_np(h), k3_out=_np(ref), k3_go=_np(go),
               k3_gx=_np(x.grad), k3_gh=_np(h.grad))

    # K4 (tests/test_correctness.py:208-214)
    x = rn(T, n, C).requires_grad_(True)
    lo = rn(T, C).requires_grad_(True)
    H = torch.randn(T, n, n, generator=g).requires_grad_(True)
    hp = torch.randn(T, n, generator=g).requires_grad_(True)
    ref = tc.TestK4FusedPostRes._ref_fwd(None, x, lo, H, hp)
    go = rn(T, n, C)
    (ref.float() * go.float()).sum().backward()
    out.update(k4_x=_np(x), k4_lo=_np(lo), k4_H=_np(H), k4_hp=_np(hp), k4_out=_np(ref),
               k4_go=_np(go), k4_gx=_np(x.grad), k4_glo=_np(lo.grad), k4_gH=_np(H.grad),
               k4_ghp=_np(hp.grad))
    return out


def _block_case(ref_pkg, tc, dtype, seed, *, T=48, C=32, outlier=False, ckpt=False):
    torch.manual_seed(seed)
    n = 4
    layer = tc._IdentityLinear(C)
    with torch.no_grad():
        layer.proj.weight.normal_(0.0, 0.02 * 8)
    blk = ref_pkg.MHCLiteBlock(n, C, layer, triton_fused=True, activation_checkpointing=ckpt)
    with torch.no_grad():
        # Move the alphas off their 0.01 init so K2's nonlinearities matter.
        blk.alpha_pre.fill_(0.7)
        blk.alpha_post.fill_(0.9)
        blk.alpha_res.fill_(1.3)
    blk = blk.to(dtype)
    blk.train()
    x = torch.randn(T, n, C)
    if outlier:
        cols = torch.randperm(C)[: max(1, C // 100 + 1)]
        x[:, :, cols] *= 100.0
    x = x.to(dtype).requires_grad_(True)
    g = torch.randn(T, n, C).to(dtype)
    out = blk._forward_pytorch(x)
    (out.float() * g.float()).sum().backward()
    with torch.no_grad():
        li, H, hpost = blk._mhc_pre_map_pytorch(x.detach())
        hpre, _, _ = blk._mhc_coeffs_pytorch(x.detach())
    res = {
        "T": T, "n": n, "C": C,
        "rms_eps": float(torch.finfo(dtype).eps),
        "x": _np(x), "g": _np(g), "out": _np(out), "grad_x": _np(x.grad),
        "alpha_pre": _np(blk.alpha_pre), "alpha_post": _np(blk.alpha_post),
        "alpha_res": _np(blk.alpha_res), "W": _np(blk.W_all.weight), "bias": _np(blk.W_all.bias),
        "perm": _np(blk.perm_mat), "Wl": _np(blk.layer.proj.weight),
        "g_alpha_pre": _np(blk.alpha_pre.grad), "g_alpha_post": _np(blk.alpha_post.grad),
        "g_alpha_res": _np(blk.alpha_res.grad), "g_W": _np(blk.W_all.weight.grad),
        "g_bias": _np(blk.W_all.bias.grad), "g_Wl": _np(blk.layer.proj.weight.grad),
        "h_pre": _np(hpre), "h_post": _np(hpost), "H_merged": _np(H), "layer_input": _np(li),
    }
    return res


def _grid_case(ref_pkg, name):
    """The reference's float32 ``_forward_pytorch`` on bf16-valued inputs and
    parameters (``block_inputs.CASES[name]``), so a bf16 path can be fed the
    very same values.  Per-token tensors are stored for ``stored_rows`` only
    (the block is token-local); parameter gradients in full, the wrapped
    layer's for 8 rows."""
    from block_inputs import CASES, block_case_inputs, stored_rows

    T, C, seed, wl_std, alphas, gelu, n_rows = CASES[name]
    inp = block_case_inputs(T, C, seed, wl_std, alphas)

    class _Layer(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.proj = torch.nn.Linear(C, C, bias=False)

        def forward(self, x):
            y = self.proj(x)
            return torch.nn.functional.gelu(y) if gelu else y

    layer = _Layer()
    blk = ref_pkg.MHCLiteBlock(4, C, layer)
    with torch.no_grad():
        for p, v in zip((blk.alpha_pre, blk.alpha_post, blk.alpha_res), inp["alphas"]):
            p.fill_(float(v))
        blk.W_all.weight.copy_(torch.from_numpy(inp["W"]))
        blk.W_all.bias.copy_(torch.from_numpy(inp["bias"]))
        layer.proj.weight.copy_(torch.from_numpy(inp["Wl"]))
    blk = blk.float().train()
    x = torch.from_numpy(inp["x"]).float().requires_grad_(True)
    out = blk._forward_pytorch(x)
    (out * torch.from_numpy(inp["g"]).float()).sum().backward()
    with torch.no_grad():
        h_pre, h_post, H = blk._mhc_coeffs_pytorch(x.detach())
        li = blk._mhc_pre_map_pytorch(x.detach())[0]
    rows = stored_rows(T, n_rows)
    wl_rows = np.arange(0, C, max(1, C // 8))[:8]
    r = lambda t: _np(t)[rows]  # noqa: E731
    return {
        "T": T, "C": C, "seed": seed, "wl_std": wl_std, "alphas": np.asarray(alphas),
        "gelu": int(gelu), "rows": rows, "wl_rows": wl_rows,
        "out": r(out), "grad_x": r(x.grad), "h_pre": r(h_pre), "h_post": r(h_post),
        "H_merged": r(H), "layer_input": r(li),
        "g_W": _np(blk.W_all.weight.grad), "g_bias": _np(blk.W_all.bias.grad),
        "g_alpha_pre": _np(blk.alpha_pre.grad), "g_alpha_post": _np(blk.alpha_post.grad),
        "g_alpha_res": _np(blk.alpha_res.grad), "g_Wl_rows": _np(layer.proj.weight.grad)[wl_rows],
    }


def _api(ref_pkg):
    lib_ops = [
        "fused_rmsnorm_project", "fused_rmsnorm_project_bwd_dx", "fused_pre_map",
        "fused_pre_map_backward", "fused_post_res", "fused_post_res_backward",
    ]
    schemas = {}
    for name in lib_ops:
        op = getattr(torch.ops.flash_mhc, name).default
        schemas[name] = str(op._schema)
    from torch._subclasses.fake_tensor import FakeTensorMode

    T, n, C = 8, 4, 16
    fake = {}
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
            fake[k] = [[list(t.shape), str(t.dtype)] for t in vs]
    blk = ref_pkg.MHCLiteBlock(4, 16, torch.nn.Linear(16, 16, bias=False))
    sd = {k: list(v.shape) for k, v in blk.state_dict().items()}
    perm, idx = ref_pkg.build_permutation_matrices(4)
    return {"schemas": schemas, "fake": fake, "state_dict": sd,
            "perm4": perm.tolist(), "perm4_identity_idx": idx,
            "torch": torch.__version__}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", required=True)
    ap.add_argument("--only-grid", action="store_true",
                    help="write only the bf16-grid block fixtures (block_inputs.CASES)")
    args = ap.parse_args()
    root = Path(args.reference_root)
    sys.path.insert(0, str(root / "src"))
    sys.path.insert(0, str(root / "tests"))
    sys.path.insert(0, str(HERE))
    sys.path.insert(0, str(HERE.parents[1]))  # the repository root, for oracle/
    import flash_mhc as ref_pkg  # the reference package
    import test_correctness as tc

    assert "flash-mhc_b200" not in ref_pkg.__file__
    torch.set_num_threads(4)
    from block_inputs import CASES

    for name in CASES:
        np.savez_compressed(HERE / f"{name}.npz", **_grid_case(ref_pkg, name))
    if args.only_grid:
        print("wrote the bf16-grid block fixtures to", HERE)
        return
    np.savez_compressed(HERE / "ops_fp32.npz", **_ops_case(tc, torch.float32, 1))
    np.savez_compressed(HERE / "ops_bf16.npz", **_ops_case(tc, torch.bfloat16, 2))
    np.savez_compressed(HERE / "block_fp32.npz", **_block_case(ref_pkg, tc, torch.float32, 3))
    np.savez_compressed(HERE / "block_bf16.npz", **_block_case(ref_pkg, tc, torch.bfloat16, 4))
    np.savez_compressed(HERE / "block_outlier_fp32.npz",
                        **_block_case(ref_pkg, tc, torch.float32, 5, T=40, C=48, outlier=True))
    ck = _block_case(ref_pkg, tc, torch.float32, 3, ckpt=True)
    nock = dict(np.load(HERE / "block_fp32.npz"))
    for k in ("out", "grad_x", "g_W", "g_bias", "g_alpha_res"):
        assert np.array_equal(ck[k], nock[k]), k  # checkpointing must not change results
    (HERE / "reference_api.json").write_text(json.dumps(_api(ref_pkg), indent=1) + "\n")
    print("wrote goldens to", HERE)


if __name__ == "__main__":
    main()
