"""Programmatic dependent launch does not change any result.

Every kernel of the library is launched with programmatic stream
serialization and waits on the preceding grid (griddepcontrol.wait) before
its first global-memory access.  The switch is read once per process, so the
same op sequence runs in two child processes, FLASH_MHC_PDL=0 and =1, and every
output must match bitwise.  The sequence chains kernels that consume each
other's outputs back to back (K1 fwd -> K2 -> K3 -> K4 -> backward), which is
where a missing wait would show.
"""

from __future__ import annotations

import os
import subprocess
import sys
import tempfile
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]

CHILD = r"""
import sys, torch
sys.path.insert(0, sys.argv[2])
import flash_mhc  # noqa: F401
ops = torch.ops.flash_mhc
torch.manual_seed(7)
T, C, n = 3000, 256, 4
dev = "cuda"
x = torch.randn(T, n, C, device=dev).bfloat16()
W = (torch.randn(32, n * C, device=dev) * 0.02).bfloat16()
lo = torch.randn(T, C, device=dev).bfloat16()
gp = torch.randn(T, 32, device=dev).bfloat16()
g3 = torch.randn(T, C, device=dev).bfloat16()
g4 = torch.randn(T, n, C, device=dev).bfloat16()
params = torch.randn(35, device=dev) * 0.5
a_pre, a_post, a_res, bias = params[0:1], params[1:2], params[2:3], params[3:35]
perm = flash_mhc.build_permutation_matrices(n)[0].to(dev)
outs = {}
for rep in range(3):
    proj, inv = ops.fused_rmsnorm_project(x.reshape(T, n * C), W)
    h_pre, h_post, H = ops.mhc_coeffs(proj, a_pre, a_post, a_res, bias, perm)
    li = ops.fused_pre_map(x, h_pre)
    out = ops.fused_post_res(x, lo, H, h_post)
    gx4, glo, gH, ghp = ops.fused_post_res_backward(g4, x, lo, H, h_post)
    gx3, gh3 = ops.fused_pre_map_backward(g3, x, h_pre)
    g_proj, gpar = ops.mhc_coeffs_backward(gh3, ghp, gH, proj, a_pre, a_post, a_res, bias, perm)
    gx1, gW = ops.fused_rmsnorm_project_backward(g_proj, x.reshape(T, n * C), W, proj, inv)
    gx = ops.mhc_grad_x_combine(gx1.view(T, n, C), g3, h_pre, gx4)
    res = dict(proj=proj, inv=inv, h_pre=h_pre, h_post=h_post, H=H, li=li, out=out, gx4=gx4,
               glo=glo, gH=gH, ghp=ghp, gx3=gx3, gh3=gh3, g_proj=g_proj, gpar=gpar, gx1=gx1,
               gW=gW, gx=gx)
    for k, v in res.items():
        outs[f"{k}{rep}"] = v.cpu()
torch.cuda.synchronize()
torch.save(outs, sys.argv[1])
"""


def _run(tmp: Path, pdl: str) -> dict:
    out = tmp / f"pdl{pdl}.pt"
    env = dict(os.environ, FLASH_MHC_PDL=pdl)
    subprocess.run([sys.executable, "-c", CHILD, str(out), str(ROOT / "flash-mhc_b200")],
                   env=env, check=True, timeout=600)
    return torch.load(out)


@pytest.mark.gpu
def test_pdl_on_and_off_give_identical_results():
    with tempfile.TemporaryDirectory() as d:
        off = _run(Path(d), "0")
        on = _run(Path(d), "1")
    assert off.keys() == on.keys()
    for k in off:
        assert torch.equal(off[k], on[k]), k
