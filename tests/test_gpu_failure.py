"""The failure path of the tensor-core kernels' bounded waits, run on a GPU
without a fault.

``fmhc_debug_k1_fwd_lost_copy`` runs the K1 forward with its first CTA arming
a pipeline stage for a copy it never issues, so the waits on that stage can
only end by expiring (about 1 s each).  The kernel must record a site code in
the device error word, release its tensor memory and return; the context must
stay usable; while the word is set the K1 backward must write grad_W as NaN
(some partials would be missing); after the word is read and cleared, the same
calls must give the results of a clean run, bit for bit.
"""

from __future__ import annotations

import time

import pytest
import torch

import flash_mhc  # noqa: F401  (registers the ops)
from flash_mhc import _native

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]

# Site codes of the K1 forward's waits that the lost copy leaves hanging
# (k1_tc.cu): the MMA issuer and the row warps wait for the stage to fill, the
# producer waits for the same stage to be released before refilling it.  The
# three waits start within microseconds of each other and each checks its
# clock every 64 polls, so whichever expires first records its site.
SITE_PROD_EMPTY, SITE_MMA_FULL, SITE_EPI_FULL = 0x101, 0x102, 0x104


def test_expired_wait_is_reported_and_the_context_stays_usable():
    T, nC = 4096, 1024
    g = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(T, nC, device="cuda", generator=g).bfloat16()
    W = (torch.randn(32, nC, device="cuda", generator=g) * 0.02).bfloat16()
    go = torch.randn(T, 32, device="cuda", generator=g).bfloat16()
    ops = torch.ops.flash_mhc
    assert _native.check_device_error() == 0

    # a clean run first
    proj, inv = ops.fused_rmsnorm_project(x, W)
    gx_ref, gW_ref = ops.fused_rmsnorm_project_backward(go, x, W, proj, inv)
    torch.cuda.synchronize()
    assert _native.check_device_error() == 0

    out = torch.zeros(T, 32, device="cuda", dtype=torch.bfloat16)
    inv_bad = torch.zeros(T, device="cuda", dtype=torch.float32)
    t0 = time.monotonic()
    _native.call("fmhc_debug_k1_fwd_lost_copy", x.data_ptr(), W.data_ptr(), out.data_ptr(),
                 inv_bad.data_ptr(), T, nC, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()  # returns: every wait is bounded
    waited = time.monotonic() - t0
    assert waited < 30.0, waited

    # While the error word is set, grad_W is NaN; grad_x is computed as usual.
    gx_err, gW_err = ops.fused_rmsnorm_project_backward(go, x, W, proj, inv)
    torch.cuda.synchronize()
    assert bool(torch.isnan(gW_err.float()).all())
    assert torch.equal(gx_err, gx_ref)

    code = _native.check_device_error()
    assert code in (SITE_PROD_EMPTY, SITE_MMA_FULL, SITE_EPI_FULL), hex(code)
    assert _native.check_device_error() == 0  # read and cleared

    # The context is usable and later calls give the clean run's bits.
    proj2, inv2 = ops.fused_rmsnorm_project(x, W)
    gx2, gW2 = ops.fused_rmsnorm_project_backward(go, x, W, proj2, inv2)
    torch.cuda.synchronize()
    assert torch.equal(proj2, proj) and torch.equal(inv2, inv)
    assert torch.equal(gx2, gx_ref) and torch.equal(gW2, gW_ref)
    assert _native.check_device_error() == 0
