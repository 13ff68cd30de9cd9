"""fmhc_k1_bwd_noalloc: the K1 backward for callers that cannot allocate.

Some callers of this library cannot allocate device memory: a C/Go/Java host
that only holds pointers handed to it, a plugin living inside another
framework's memory pool, a serving runtime that reserved all of HBM up front,
or a latency-critical path where cudaMalloc's implicit synchronisation is not
allowed.  For them the library exports fmhc_k1_bwd_noalloc, which takes the
same inputs and outputs as fmhc_k1_bwd but uses a fixed 32 MiB scratch array
built into the library instead of a caller workspace.

This test calls both entry points through the C ABI (ctypes) on the same
inputs and checks that the allocation-free one matches the workspace one within
the tolerances the other GPU tests use (bf16: 2e-2 + 1e-2*|ref|), on two calls
in a row (the second reuses whatever the first left in the shared scratch).
Before the checked calls of every case, one call on unrelated inputs of the
largest shape fills the scratch with other values, so a read of a scratch
value the checked call did not write would show, whichever case runs alone.
It is collected last on purpose (file name), so a failure here never hides
another test's result.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from flash_mhc import _native

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device"),
]

_vp, _i64 = ctypes.c_void_p, ctypes.c_int64
ATOL, RTOL = 2e-2, 1e-2


def _lib():
    L = _native.lib()
    fn = L.fmhc_k1_bwd_noalloc
    fn.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]
    fn.restype = ctypes.c_int
    return L


def _inputs(T, nC, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, nC, device="cuda", generator=g).bfloat16()
    W = (torch.randn(32, nC, device="cuda", generator=g) * 0.02).bfloat16()
    go = torch.randn(T, 32, device="cuda", generator=g).bfloat16()
    proj, inv = torch.ops.flash_mhc.fused_rmsnorm_project(x, W)
    return go, x, W, proj, inv


def _with_workspace(L, go, x, W, proj, inv):
    T, nC = x.shape
    gx = torch.empty_like(x)
    gW = torch.empty_like(W)
    ws_bytes = int(L.fmhc_k1_bwd_workspace_size(T, nC, 32))
    ws = torch.empty(max(ws_bytes, 1), device="cuda", dtype=torch.uint8)
    st = L.fmhc_k1_bwd(go.data_ptr(), x.data_ptr(), W.data_ptr(), proj.data_ptr(),
                       inv.data_ptr(), gx.data_ptr(), gW.data_ptr(), ws.data_ptr(), ws_bytes,
                       T, nC, 32, torch.cuda.current_stream().cuda_stream)
    assert st == 0, L.fmhc_last_error().decode()
    return gx, gW


def _no_alloc(L, go, x, W, proj, inv):
    T, nC = x.shape
    gx = torch.empty_like(x)
    gW = torch.empty_like(W)
    st = L.fmhc_k1_bwd_noalloc(go.data_ptr(), x.data_ptr(), W.data_ptr(), proj.data_ptr(),
                               inv.data_ptr(), gx.data_ptr(), gW.data_ptr(), T, nC, 32,
                               torch.cuda.current_stream().cuda_stream)
    assert st == 0, L.fmhc_last_error().decode()
    return gx, gW


def _fill_scratch(L):
    """One call on unrelated inputs of the largest shape (its grad_W partials
    cover the most scratch), leaving their values in the shared array."""
    go, x, W, proj, inv = _inputs(65536, 4096, seed=999)
    go.mul_(3.0)
    _no_alloc(L, go, x, W, proj, inv)
    torch.cuda.synchronize()


@pytest.mark.parametrize("T,nC", [(65536, 4096), (4097, 1024), (300, 400)])
def test_no_alloc_matches_workspace_entry_point(T, nC):
    import flash_mhc  # noqa: F401  (registers the ops used to make inputs)

    L = _lib()
    go, x, W, proj, inv = _inputs(T, nC, seed=T + nC)
    ref_gx, ref_gW = _with_workspace(L, go, x, W, proj, inv)
    _fill_scratch(L)
    for _ in range(2):  # two calls in a row share the scratch array
        gx, gW = _no_alloc(L, go, x, W, proj, inv)
        torch.cuda.synchronize()
        torch.testing.assert_close(gx.float(), ref_gx.float(), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(gW.float(), ref_gW.float(), atol=ATOL, rtol=RTOL)
        # The reductions use a fixed order, so the bits agree as well.
        assert torch.equal(gx, ref_gx) and torch.equal(gW, ref_gW)
    assert _native.check_device_error() == 0


def test_no_alloc_rejects_sizes_above_its_scratch():
    L = _lib()
    L.fmhc_k1_bwd_workspace_size.argtypes = [_i64, _i64, _i64]
    L.fmhc_k1_bwd_workspace_size.restype = _i64
    # nC = 16400 is not a multiple of 128, so this shape takes the CUDA-core
    # path, whose workspace (16 x 32 x nC f32) is above the 32 MiB scratch.
    # The size is checked first: the call below hands the entry point a
    # 32-byte dummy buffer and must be rejected before any launch.
    T, nC = 1 << 22, 16400
    assert L.fmhc_k1_bwd_workspace_size(T, nC, 32) > (32 << 20)
    dummy = torch.empty(16, device="cuda", dtype=torch.bfloat16)
    p = dummy.data_ptr()
    st = L.fmhc_k1_bwd_noalloc(p, p, p, p, p, p, p, T, nC, 32, None)
    assert st == 6  # FMHC_ERR_WORKSPACE, before any launch
    assert "maximum" in L.fmhc_last_error().decode()
