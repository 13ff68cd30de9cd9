"""torch.library custom ops of mHC-lite, backed by the sm_100a C-ABI library.

The op namespace, the six schemas, the fake (meta) implementations and the
autograd formulas are those of the reference (src/flash_mhc/ops.py:22-41,
145-202, 670-714), so this module is a drop-in: ``torch.ops.flash_mhc.*``
calls, ``torch.compile`` tracing through the fakes, and autograd all behave
as before.  The CUDA implementations allocate the outputs with torch, pass raw
pointers and the current CUDA stream to ``libflashmhc_sm100.so`` and raise on
a non-zero status.  There is no CPU kernel (as in the reference: the ops raise
on CPU tensors) and no fallback when the library is missing.

Added beyond the reference: ``fused_rmsnorm_project_backward`` computes K1's
grad_x AND grad_W in one op; K1's autograd formula uses it instead of the
reference's separate cuBLAS matmul (src/flash_mhc/ops.py:683-684).
"""

from __future__ import annotations

import os
import threading
from contextlib import contextmanager

import torch
import torch.library

from . import _native

_lib = torch.library.Library("flash_mhc", "DEF")

_lib.define(
    "fused_rmsnorm_project(Tensor x_flat, Tensor W) -> (Tensor out, Tensor inv_rms)"
)
_lib.define(
    "fused_rmsnorm_project_bwd_dx(Tensor grad_out, Tensor x_flat, Tensor W, Tensor proj_out, Tensor inv_rms) -> Tensor grad_x"
)
_lib.define("fused_pre_map(Tensor x_streams, Tensor h_pre) -> Tensor out")
_lib.define(
    "fused_pre_map_backward(Tensor grad_out, Tensor x_streams, Tensor h_pre) -> (Tensor grad_x, Tensor grad_h_pre)"
)
_lib.define(
    "fused_post_res(Tensor x_streams, Tensor layer_output, Tensor H_merged, Tensor h_post) -> Tensor out"
)
_lib.define(
    "fused_post_res_backward(Tensor grad_out, Tensor x_streams, Tensor layer_output, Tensor H_merged, Tensor h_post) -> (Tensor grad_x, Tensor grad_layer_output, Tensor grad_H_merged, Tensor grad_h_post)"
)
# Not in the reference: K1 grad_x and grad_W together.
_lib.define(
    "fused_rmsnorm_project_backward(Tensor grad_out, Tensor x_flat, Tensor W, Tensor proj_out, Tensor inv_rms) -> (Tensor grad_x, Tensor grad_W)"
)
# Not in the reference: K2 (the coefficient math of block.py:150-170) as one
# kernel each way; outputs are the f32 coefficients K3/K4 consume.
_lib.define(
    "mhc_coeffs(Tensor proj, Tensor alpha_pre, Tensor alpha_post, Tensor alpha_res, Tensor bias, Tensor perm) -> (Tensor h_pre, Tensor h_post, Tensor H_merged)"
)
# Not in the reference: the block's pre-map forward in one call -- K1 with K2
# in its epilogue, then K3 (at few tokens all three in one kernel); replaces
# block.py:150-177 (_mhc_coeffs_triton + _mhc_pre_map_triton).
_lib.define(
    "mhc_pre_forward(Tensor x_streams, Tensor W, Tensor alpha_pre, Tensor alpha_post, Tensor alpha_res, Tensor bias, Tensor perm) -> (Tensor layer_input, Tensor proj, Tensor inv_rms, Tensor h_pre, Tensor h_post, Tensor H_merged)"
)
# Not in the reference: pieces of the fused block backward.
_lib.define("pre_map_grad_h(Tensor grad_out, Tensor x_streams, Tensor h_pre) -> Tensor grad_h_pre")
_lib.define(
    "mhc_grad_x_combine(Tensor gx1, Tensor grad_layer_input, Tensor h_pre, Tensor? gx4) -> Tensor grad_x"
)
# K4 backward without its grad_x, and the combination that forms K4's grad_x
# from K4's upstream gradient instead (one (T, n, C) write and read fewer).
_lib.define(
    "post_res_grad_params(Tensor grad_out, Tensor x_streams, Tensor layer_output, Tensor H_merged, Tensor h_post) -> (Tensor grad_layer_output, Tensor grad_H_merged, Tensor grad_h_post)"
)
_lib.define(
    "mhc_grad_x_combine_post(Tensor gx1, Tensor grad_layer_input, Tensor h_pre, Tensor grad_out, Tensor H_merged) -> Tensor grad_x"
)
_lib.define(
    "mhc_coeffs_backward(Tensor grad_h_pre, Tensor grad_h_post, Tensor grad_H_merged, Tensor proj, Tensor alpha_pre, Tensor alpha_post, Tensor alpha_res, Tensor bias, Tensor perm) -> (Tensor grad_proj, Tensor grad_params)"
)
# The same with one gradient per parameter, in the parameter's shape and dtype.
_lib.define(
    "mhc_coeffs_backward_split(Tensor grad_h_pre, Tensor grad_h_post, Tensor grad_H_merged, Tensor proj, Tensor alpha_pre, Tensor alpha_post, Tensor alpha_res, Tensor bias, Tensor perm) -> (Tensor grad_proj, Tensor grad_alpha_pre, Tensor grad_alpha_post, Tensor grad_alpha_res, Tensor grad_bias)"
)

# ---------------------------------------------------------------------------
# Autotune controls.  The reference exposes a thread-local context manager and
# environment switches for its Triton autotuner (src/flash_mhc/ops.py:44-68).
# The CUDA kernels here have fixed, shape-derived launch configurations and no
# runtime search; the API is kept so callers keep working, and it changes
# nothing.
# ---------------------------------------------------------------------------
_AUTOTUNE_CONTROL = threading.local()


def _autotune_disable_depth() -> int:
    return int(getattr(_AUTOTUNE_CONTROL, "disable_depth", 0))


@contextmanager
def disable_autotune_temporarily():
    """Kept for API compatibility; launch configurations are fixed (no autotune)."""
    _AUTOTUNE_CONTROL.disable_depth = _autotune_disable_depth() + 1
    try:
        yield
    finally:
        _AUTOTUNE_CONTROL.disable_depth = max(0, _autotune_disable_depth() - 1)


def _autotune_enabled() -> bool:
    """Mirrors the reference switch (FLASH_MHC_TRITON_AUTOTUNE); informational only."""
    v = os.getenv("FLASH_MHC_TRITON_AUTOTUNE", "1").strip().lower()
    return v not in {"0", "false", "off", "no"} and _autotune_disable_depth() == 0


# ---------------------------------------------------------------------------
# Fake implementations (shapes/dtypes identical to src/flash_mhc/ops.py:145-202)
# ---------------------------------------------------------------------------


@torch.library.register_fake("flash_mhc::fused_rmsnorm_project")
def _fused_rmsnorm_project_fake(x_flat: torch.Tensor, W: torch.Tensor):
    T = x_flat.shape[0]
    D_out = W.shape[0]
    out = torch.empty((T, D_out), device=x_flat.device, dtype=x_flat.dtype)
    inv_rms = torch.empty((T,), device=x_flat.device, dtype=torch.float32)
    return out, inv_rms


@torch.library.register_fake("flash_mhc::fused_rmsnorm_project_bwd_dx")
def _fused_rmsnorm_project_bwd_dx_fake(grad_out, x_flat, W, proj_out, inv_rms):
    return torch.empty_like(x_flat)


@torch.library.register_fake("flash_mhc::fused_rmsnorm_project_backward")
def _fused_rmsnorm_project_backward_fake(grad_out, x_flat, W, proj_out, inv_rms):
    return torch.empty_like(x_flat), torch.empty_like(W, dtype=x_flat.dtype)


@torch.library.register_fake("flash_mhc::mhc_coeffs")
def _mhc_coeffs_fake(proj, alpha_pre, alpha_post, alpha_res, bias, perm):
    T = proj.shape[0]
    f = dict(device=proj.device, dtype=torch.float32)
    return torch.empty((T, 4), **f), torch.empty((T, 4), **f), torch.empty((T, 4, 4), **f)


@torch.library.register_fake("flash_mhc::mhc_pre_forward")
def _mhc_pre_forward_fake(x_streams, W, alpha_pre, alpha_post, alpha_res, bias, perm):
    T, n, C = x_streams.shape
    f = dict(device=x_streams.device, dtype=torch.float32)
    return (torch.empty((T, C), device=x_streams.device, dtype=x_streams.dtype),
            torch.empty((T, W.shape[0]), device=x_streams.device, dtype=x_streams.dtype),
            torch.empty((T,), **f), torch.empty((T, 4), **f), torch.empty((T, 4), **f),
            torch.empty((T, 4, 4), **f))


@torch.library.register_fake("flash_mhc::mhc_coeffs_backward")
def _mhc_coeffs_backward_fake(grad_h_pre, grad_h_post, grad_H_merged, proj, alpha_pre,
                              alpha_post, alpha_res, bias, perm):
    return torch.empty_like(proj), torch.empty((35,), device=proj.device, dtype=torch.float32)


@torch.library.register_fake("flash_mhc::mhc_coeffs_backward_split")
def _mhc_coeffs_backward_split_fake(grad_h_pre, grad_h_post, grad_H_merged, proj, alpha_pre,
                                    alpha_post, alpha_res, bias, perm):
    return (torch.empty_like(proj), torch.empty_like(alpha_pre), torch.empty_like(alpha_post),
            torch.empty_like(alpha_res), torch.empty_like(bias))


@torch.library.register_fake("flash_mhc::pre_map_grad_h")
def _pre_map_grad_h_fake(grad_out, x_streams, h_pre):
    return torch.empty_like(h_pre, dtype=torch.float32)


@torch.library.register_fake("flash_mhc::mhc_grad_x_combine")
def _mhc_grad_x_combine_fake(gx1, grad_layer_input, h_pre, gx4):
    return torch.empty_like(gx1)


@torch.library.register_fake("flash_mhc::post_res_grad_params")
def _post_res_grad_params_fake(grad_out, x_streams, layer_output, H_merged, h_post):
    T, n, C = x_streams.shape
    return (x_streams.new_empty((T, C)),
            x_streams.new_empty((T, n, n), dtype=torch.float32),
            x_streams.new_empty((T, n), dtype=torch.float32))


@torch.library.register_fake("flash_mhc::mhc_grad_x_combine_post")
def _mhc_grad_x_combine_post_fake(gx1, grad_layer_input, h_pre, grad_out, H_merged):
    return torch.empty_like(gx1)


@torch.library.register_fake("flash_mhc::fused_pre_map")
def _fused_pre_map_fake(x_streams: torch.Tensor, h_pre: torch.Tensor):
    T, _, C = x_streams.shape
    return torch.empty((T, C), device=x_streams.device, dtype=x_streams.dtype)


@torch.library.register_fake("flash_mhc::fused_pre_map_backward")
def _fused_pre_map_backward_fake(grad_out, x_streams, h_pre):
    grad_x = torch.empty_like(x_streams)
    grad_h_pre = torch.empty_like(h_pre, dtype=torch.float32)
    return grad_x, grad_h_pre


@torch.library.register_fake("flash_mhc::fused_post_res")
def _fused_post_res_fake(x_streams, layer_output, H_merged, h_post):
    return torch.empty_like(x_streams)


@torch.library.register_fake("flash_mhc::fused_post_res_backward")
def _fused_post_res_backward_fake(grad_out, x_streams, layer_output, H_merged, h_post):
    grad_x = torch.empty_like(x_streams)
    grad_layer_output = torch.empty_like(layer_output)
    grad_H_merged = torch.empty_like(H_merged, dtype=torch.float32)
    grad_h_post = torch.empty_like(h_post, dtype=torch.float32)
    return grad_x, grad_layer_output, grad_H_merged, grad_h_post


# ---------------------------------------------------------------------------
# CUDA implementations
# ---------------------------------------------------------------------------


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _bf16(name: str, t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        raise ValueError(f"flash_mhc: {name} must be bfloat16 (got {t.dtype})")
    return t.contiguous()


def _coef(t: torch.Tensor) -> torch.Tensor:
    """Small f32 coefficient tensors: contiguous, float32, 16-byte aligned."""
    t = t.to(torch.float32).contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def _n4(op: str, n: int) -> None:
    if n != 4:
        raise ValueError(f"flash_mhc::{op} currently supports n=4 only")


class _on_device:
    """Make ``t``'s device current for the duration of a C-ABI call."""

    __slots__ = ("idx", "prev")

    def __init__(self, t: torch.Tensor):
        self.idx = t.device.index

    def __enter__(self):
        self.prev = torch.cuda.current_device()
        if self.idx is not None and self.idx != self.prev:
            torch.cuda.set_device(self.idx)

    def __exit__(self, *exc):
        if self.idx is not None and self.idx != self.prev:
            torch.cuda.set_device(self.prev)


@torch.library.impl(_lib, "fused_rmsnorm_project", "CUDA")
def _fused_rmsnorm_project_cuda(x_flat: torch.Tensor, W: torch.Tensor):
    x_flat = _bf16("x_flat", x_flat)
    W = _bf16("W", W)
    T, nC = x_flat.shape
    D_out = W.shape[0]
    if W.shape[1] != nC:
        raise ValueError(f"flash_mhc::fused_rmsnorm_project: W is {tuple(W.shape)}, x_flat has nC={nC}")
    out = torch.empty((T, D_out), device=x_flat.device, dtype=x_flat.dtype)
    inv_rms = torch.empty((T,), device=x_flat.device, dtype=torch.float32)
    with _on_device(x_flat):
        _native.call("fmhc_k1_fwd", x_flat.data_ptr(), W.data_ptr(), out.data_ptr(),
                     inv_rms.data_ptr(), T, nC, D_out, _stream(x_flat))
    return out, inv_rms


@torch.library.impl(_lib, "fused_rmsnorm_project_bwd_dx", "CUDA")
def _fused_rmsnorm_project_bwd_dx_cuda(grad_out, x_flat, W, proj_out, inv_rms):
    grad_out = _bf16("grad_out", grad_out)
    x_flat = _bf16("x_flat", x_flat)
    W = _bf16("W", W)
    proj_out = _bf16("proj_out", proj_out)
    inv_rms = inv_rms.to(torch.float32).contiguous()
    T, nC = x_flat.shape
    D_out = W.shape[0]
    grad_x = torch.empty_like(x_flat)
    with _on_device(x_flat):
        _native.call("fmhc_k1_bwd_dx", grad_out.data_ptr(), x_flat.data_ptr(), W.data_ptr(),
                     proj_out.data_ptr(), inv_rms.data_ptr(), grad_x.data_ptr(), T, nC, D_out,
                     _stream(x_flat))
    return grad_x


@torch.library.impl(_lib, "fused_rmsnorm_project_backward", "CUDA")
def _fused_rmsnorm_project_backward_cuda(grad_out, x_flat, W, proj_out, inv_rms):
    grad_out = _bf16("grad_out", grad_out)
    x_flat = _bf16("x_flat", x_flat)
    W = _bf16("W", W)
    proj_out = _bf16("proj_out", proj_out)
    inv_rms = inv_rms.to(torch.float32).contiguous()
    T, nC = x_flat.shape
    D_out = W.shape[0]
    grad_x = torch.empty_like(x_flat)
    grad_W = torch.empty((D_out, nC), device=x_flat.device, dtype=x_flat.dtype)
    with _on_device(x_flat):
        ws_bytes = _native.workspace_size_k1_bwd(T, nC, D_out)
        ws = torch.empty(max(ws_bytes, 1), device=x_flat.device, dtype=torch.uint8)
        _native.call("fmhc_k1_bwd", grad_out.data_ptr(), x_flat.data_ptr(), W.data_ptr(),
                     proj_out.data_ptr(), inv_rms.data_ptr(), grad_x.data_ptr(),
                     grad_W.data_ptr(), ws.data_ptr(), ws_bytes, T, nC, D_out, _stream(x_flat))
    return grad_x, grad_W


def _k2_params(proj, alpha_pre, alpha_post, alpha_res, bias, perm):
    if proj.dim() != 2 or proj.shape[1] != 32:
        raise ValueError(f"flash_mhc::mhc_coeffs: proj must be (T, 32) (n=4), got {tuple(proj.shape)}")
    if bias.numel() != 32 or perm.shape != (24, 16):
        raise ValueError("flash_mhc::mhc_coeffs: bias must have 32 entries and perm be (24, 16)")
    params = torch.cat([alpha_pre.reshape(-1)[:1], alpha_post.reshape(-1)[:1],
                        alpha_res.reshape(-1)[:1], bias.reshape(-1)]).to(torch.float32).contiguous()
    return _bf16("proj", proj), params, perm.to(torch.float32).contiguous()


_K2_DTYPES = {torch.float32: 0, torch.bfloat16: 1}  # FMHC_DTYPE_F32, FMHC_DTYPE_BF16


def _k2_typed_args(alpha_pre, alpha_post, alpha_res, bias, perm):
    """Pointer arguments of the typed K2 entries, and the tensors they point into.

    f32 or bf16 parameters of one dtype are passed as they are (the kernel
    reads them in their own dtype); anything else is packed to f32 first."""
    if bias.numel() != 32 or perm.shape != (24, 16):
        raise ValueError("flash_mhc::mhc_coeffs: bias must have 32 entries and perm be (24, 16)")
    pdt, qdt = _K2_DTYPES.get(bias.dtype), _K2_DTYPES.get(perm.dtype)
    same = all(a.dtype == bias.dtype for a in (alpha_pre, alpha_post, alpha_res))
    if pdt is None or qdt is None or not same:
        params = torch.cat([alpha_pre.reshape(-1)[:1], alpha_post.reshape(-1)[:1],
                            alpha_res.reshape(-1)[:1], bias.reshape(-1)]).to(torch.float32).contiguous()
        perm = perm.to(torch.float32).contiguous()
        p = params.data_ptr()
        return (p, p + 4, p + 8, p + 12, 0, perm.data_ptr(), 0), (params, perm)
    a_pre, a_post, a_res = (a.contiguous() for a in (alpha_pre, alpha_post, alpha_res))
    bias, perm = bias.contiguous(), perm.contiguous()
    return ((a_pre.data_ptr(), a_post.data_ptr(), a_res.data_ptr(), bias.data_ptr(), pdt,
             perm.data_ptr(), qdt), (a_pre, a_post, a_res, bias, perm))


@torch.library.impl(_lib, "mhc_coeffs", "CUDA")
def _mhc_coeffs_cuda(proj, alpha_pre, alpha_post, alpha_res, bias, perm):
    if proj.dim() != 2 or proj.shape[1] != 32:
        raise ValueError(f"flash_mhc::mhc_coeffs: proj must be (T, 32) (n=4), got {tuple(proj.shape)}")
    proj = _bf16("proj", proj)
    args, _keep = _k2_typed_args(alpha_pre, alpha_post, alpha_res, bias, perm)
    T = proj.shape[0]
    f = dict(device=proj.device, dtype=torch.float32)
    h_pre, h_post, H = torch.empty((T, 4), **f), torch.empty((T, 4), **f), torch.empty((T, 4, 4), **f)
    with _on_device(proj):
        _native.call("fmhc_k2_fwd_typed", proj.data_ptr(), *args, h_pre.data_ptr(),
                     h_post.data_ptr(), H.data_ptr(), T, _stream(proj))
    return h_pre, h_post, H


@torch.library.impl(_lib, "mhc_pre_forward", "CUDA")
def _mhc_pre_forward_cuda(x_streams, W, alpha_pre, alpha_post, alpha_res, bias, perm):
    T, n, C = x_streams.shape
    _n4("mhc_pre_forward", n)
    x_streams = _bf16("x_streams", x_streams)
    W = _bf16("W", W)
    if tuple(W.shape) != (32, n * C):
        raise ValueError(f"flash_mhc::mhc_pre_forward: W must be (32, {n * C}), got {tuple(W.shape)}")
    args, _keep = _k2_typed_args(alpha_pre, alpha_post, alpha_res, bias, perm)
    dev, dt = x_streams.device, x_streams.dtype
    f = dict(device=dev, dtype=torch.float32)
    layer_input = torch.empty((T, C), device=dev, dtype=dt)
    proj = torch.empty((T, 32), device=dev, dtype=dt)
    inv_rms = torch.empty((T,), **f)
    h_pre, h_post, H = torch.empty((T, 4), **f), torch.empty((T, 4), **f), torch.empty((T, 4, 4), **f)
    with _on_device(x_streams):
        _native.call("fmhc_mhc_pre_fwd", x_streams.data_ptr(), W.data_ptr(), *args,
                     proj.data_ptr(), inv_rms.data_ptr(), h_pre.data_ptr(), h_post.data_ptr(),
                     H.data_ptr(), layer_input.data_ptr(), T, n, C, _stream(x_streams))
    return layer_input, proj, inv_rms, h_pre, h_post, H


@torch.library.impl(_lib, "mhc_coeffs_backward", "CUDA")
def _mhc_coeffs_backward_cuda(grad_h_pre, grad_h_post, grad_H_merged, proj, alpha_pre,
                              alpha_post, alpha_res, bias, perm):
    proj, params, perm = _k2_params(proj, alpha_pre, alpha_post, alpha_res, bias, perm)
    T = proj.shape[0]
    g1, g2, g3 = _coef(grad_h_pre), _coef(grad_h_post), _coef(grad_H_merged)
    grad_proj = torch.empty_like(proj)
    grad_params = torch.empty((35,), device=proj.device, dtype=torch.float32)
    with _on_device(proj):
        ws_bytes = int(_native.lib().fmhc_k2_bwd_workspace_size(T))
        ws = torch.empty(max(ws_bytes, 1), device=proj.device, dtype=torch.uint8)
        _native.call("fmhc_k2_bwd", proj.data_ptr(), params.data_ptr(), perm.data_ptr(),
                     g1.data_ptr(), g2.data_ptr(), g3.data_ptr(), grad_proj.data_ptr(),
                     grad_params.data_ptr(), ws.data_ptr(), ws_bytes, T, _stream(proj))
    return grad_proj, grad_params


@torch.library.impl(_lib, "mhc_coeffs_backward_split", "CUDA")
def _mhc_coeffs_backward_split_cuda(grad_h_pre, grad_h_post, grad_H_merged, proj, alpha_pre,
                                    alpha_post, alpha_res, bias, perm):
    pdt, qdt = _K2_DTYPES.get(bias.dtype), _K2_DTYPES.get(perm.dtype)
    same = all(a.dtype == bias.dtype for a in (alpha_pre, alpha_post, alpha_res))
    if pdt is None or qdt is None or not same or proj.dim() != 2 or proj.shape[1] != 32 \
            or bias.numel() != 32 or perm.shape != (24, 16) \
            or any(a.numel() != 1 for a in (alpha_pre, alpha_post, alpha_res)):
        # Other dtypes or shapes: the packed f32 path, then split and cast.
        g_proj, gp = _mhc_coeffs_backward_cuda(grad_h_pre, grad_h_post, grad_H_merged, proj,
                                               alpha_pre, alpha_post, alpha_res, bias, perm)
        return (g_proj, gp[0:1].view_as(alpha_pre).to(alpha_pre.dtype),
                gp[1:2].view_as(alpha_post).to(alpha_post.dtype),
                gp[2:3].view_as(alpha_res).to(alpha_res.dtype),
                gp[3:35].view_as(bias).to(bias.dtype))
    proj = _bf16("proj", proj)
    a_pre, a_post, a_res = (a.contiguous() for a in (alpha_pre, alpha_post, alpha_res))
    bias, perm = bias.contiguous(), perm.contiguous()
    T = proj.shape[0]
    g1, g2, g3 = _coef(grad_h_pre), _coef(grad_h_post), _coef(grad_H_merged)
    grad_proj = torch.empty_like(proj)
    outs = [torch.empty_like(t) for t in (a_pre, a_post, a_res, bias)]
    with _on_device(proj):
        ws_bytes = int(_native.lib().fmhc_k2_bwd_workspace_size(T))
        ws = torch.empty(max(ws_bytes, 1), device=proj.device, dtype=torch.uint8)
        _native.call("fmhc_k2_bwd_typed", proj.data_ptr(), a_pre.data_ptr(), a_post.data_ptr(),
                     a_res.data_ptr(), bias.data_ptr(), pdt, perm.data_ptr(), qdt,
                     g1.data_ptr(), g2.data_ptr(), g3.data_ptr(), grad_proj.data_ptr(),
                     *(o.data_ptr() for o in outs), ws.data_ptr(), ws_bytes, T, _stream(proj))
    return (grad_proj, *outs)


@torch.library.impl(_lib, "fused_pre_map", "CUDA")
def _fused_pre_map_cuda(x_streams: torch.Tensor, h_pre: torch.Tensor):
    T, n, C = x_streams.shape
    _n4("fused_pre_map", n)
    x_streams = _bf16("x_streams", x_streams)
    h_pre = _coef(h_pre)
    out = torch.empty((T, C), device=x_streams.device, dtype=x_streams.dtype)
    with _on_device(x_streams):
        _native.call("fmhc_k3_fwd", x_streams.data_ptr(), h_pre.data_ptr(), out.data_ptr(),
                     T, n, C, _stream(x_streams))
    return out


@torch.library.impl(_lib, "fused_pre_map_backward", "CUDA")
def _fused_pre_map_backward_cuda(grad_out, x_streams, h_pre):
    T, n, C = x_streams.shape
    _n4("fused_pre_map_backward", n)
    grad_out = _bf16("grad_out", grad_out)
    x_streams = _bf16("x_streams", x_streams)
    h_pre = _coef(h_pre)
    grad_x = torch.empty_like(x_streams)
    grad_h_pre = torch.empty((T, n), device=x_streams.device, dtype=torch.float32)
    with _on_device(x_streams):
        _native.call("fmhc_k3_bwd", grad_out.data_ptr(), x_streams.data_ptr(), h_pre.data_ptr(),
                     grad_x.data_ptr(), grad_h_pre.data_ptr(), T, n, C, _stream(x_streams))
    return grad_x, grad_h_pre


@torch.library.impl(_lib, "pre_map_grad_h", "CUDA")
def _pre_map_grad_h_cuda(grad_out, x_streams, h_pre):
    T, n, C = x_streams.shape
    _n4("pre_map_grad_h", n)
    grad_out = _bf16("grad_out", grad_out)
    x_streams = _bf16("x_streams", x_streams)
    h_pre = _coef(h_pre)
    grad_h_pre = torch.empty((T, n), device=x_streams.device, dtype=torch.float32)
    with _on_device(x_streams):
        _native.call("fmhc_k3_bwd", grad_out.data_ptr(), x_streams.data_ptr(), h_pre.data_ptr(),
                     None, grad_h_pre.data_ptr(), T, n, C, _stream(x_streams))
    return grad_h_pre


@torch.library.impl(_lib, "mhc_grad_x_combine", "CUDA")
def _mhc_grad_x_combine_cuda(gx1, grad_layer_input, h_pre, gx4):
    T, n, C = gx1.shape
    _n4("mhc_grad_x_combine", n)
    gx1 = _bf16("gx1", gx1)
    gli = _bf16("grad_layer_input", grad_layer_input)
    h_pre = _coef(h_pre)
    gx4 = None if gx4 is None else _bf16("gx4", gx4)
    grad_x = torch.empty_like(gx1)
    with _on_device(gx1):
        _native.call("fmhc_mhc_grad_x_combine", gx1.data_ptr(), gli.data_ptr(), h_pre.data_ptr(),
                     None if gx4 is None else gx4.data_ptr(), grad_x.data_ptr(), T, n, C,
                     _stream(gx1))
    return grad_x


@torch.library.impl(_lib, "mhc_grad_x_combine_post", "CUDA")
def _mhc_grad_x_combine_post_cuda(gx1, grad_layer_input, h_pre, grad_out, H_merged):
    T, n, C = gx1.shape
    _n4("mhc_grad_x_combine_post", n)
    gx1 = _bf16("gx1", gx1)
    gli = _bf16("grad_layer_input", grad_layer_input)
    h_pre = _coef(h_pre)
    grad_out = _bf16("grad_out", grad_out)
    H_merged = _coef(H_merged)
    grad_x = torch.empty_like(gx1)
    with _on_device(gx1):
        _native.call("fmhc_mhc_grad_x_combine_post", gx1.data_ptr(), gli.data_ptr(),
                     h_pre.data_ptr(), grad_out.data_ptr(), H_merged.data_ptr(),
                     grad_x.data_ptr(), T, n, C, _stream(gx1))
    return grad_x


@torch.library.impl(_lib, "post_res_grad_params", "CUDA")
def _post_res_grad_params_cuda(grad_out, x_streams, layer_output, H_merged, h_post):
    T, n, C = x_streams.shape
    _n4("post_res_grad_params", n)
    grad_out = _bf16("grad_out", grad_out)
    x_streams = _bf16("x_streams", x_streams)
    layer_output = _bf16("layer_output", layer_output)
    H_merged = _coef(H_merged)
    h_post = _coef(h_post)
    grad_layer_output = torch.empty((T, C), device=x_streams.device, dtype=x_streams.dtype)
    grad_H = torch.empty((T, n, n), device=x_streams.device, dtype=torch.float32)
    grad_hp = torch.empty((T, n), device=x_streams.device, dtype=torch.float32)
    with _on_device(x_streams):
        _native.call("fmhc_k4_bwd", grad_out.data_ptr(), x_streams.data_ptr(),
                     layer_output.data_ptr(), H_merged.data_ptr(), h_post.data_ptr(),
                     None, grad_layer_output.data_ptr(), grad_H.data_ptr(),
                     grad_hp.data_ptr(), T, n, C, _stream(x_streams))
    return grad_layer_output, grad_H, grad_hp


@torch.library.impl(_lib, "fused_post_res", "CUDA")
def _fused_post_res_cuda(x_streams, layer_output, H_merged, h_post):
    T, n, C = x_streams.shape
    _n4("fused_post_res", n)
    x_streams = _bf16("x_streams", x_streams)
    layer_output = _bf16("layer_output", layer_output)
    H_merged = _coef(H_merged)
    h_post = _coef(h_post)
    out = torch.empty_like(x_streams)
    with _on_device(x_streams):
        _native.call("fmhc_k4_fwd", x_streams.data_ptr(), layer_output.data_ptr(),
                     H_merged.data_ptr(), h_post.data_ptr(), out.data_ptr(), T, n, C,
                     _stream(x_streams))
    return out


@torch.library.impl(_lib, "fused_post_res_backward", "CUDA")
def _fused_post_res_backward_cuda(grad_out, x_streams, layer_output, H_merged, h_post):
    T, n, C = x_streams.shape
    _n4("fused_post_res_backward", n)
    grad_out = _bf16("grad_out", grad_out)
    x_streams = _bf16("x_streams", x_streams)
    layer_output = _bf16("layer_output", layer_output)
    H_merged = _coef(H_merged)
    h_post = _coef(h_post)
    grad_x = torch.empty_like(x_streams)
    grad_layer_output = torch.empty((T, C), device=x_streams.device, dtype=x_streams.dtype)
    grad_H = torch.empty((T, n, n), device=x_streams.device, dtype=torch.float32)
    grad_hp = torch.empty((T, n), device=x_streams.device, dtype=torch.float32)
    with _on_device(x_streams):
        _native.call("fmhc_k4_bwd", grad_out.data_ptr(), x_streams.data_ptr(),
                     layer_output.data_ptr(), H_merged.data_ptr(), h_post.data_ptr(),
                     grad_x.data_ptr(), grad_layer_output.data_ptr(), grad_H.data_ptr(),
                     grad_hp.data_ptr(), T, n, C, _stream(x_streams))
    return grad_x, grad_layer_output, grad_H, grad_hp


# ---------------------------------------------------------------------------
# Autograd (src/flash_mhc/ops.py:670-714): inputs and outputs are saved; K1's
# grad w.r.t. inv_rms is ignored, as in the reference.
# ---------------------------------------------------------------------------


def _setup_save_inputs_outputs(ctx, inputs, output):
    if isinstance(output, tuple):
        ctx.save_for_backward(*inputs, *output)
    else:
        ctx.save_for_backward(*inputs, output)


def _fused_rmsnorm_project_backward(ctx, grad_out, grad_inv_rms):
    x_flat, W, proj_out, inv_rms = ctx.saved_tensors
    need_x, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
    if need_w:
        grad_x, grad_W = torch.ops.flash_mhc.fused_rmsnorm_project_backward(
            grad_out, x_flat, W, proj_out, inv_rms)
        return (grad_x if need_x else None), grad_W
    grad_x = torch.ops.flash_mhc.fused_rmsnorm_project_bwd_dx(
        grad_out, x_flat, W, proj_out, inv_rms)
    return grad_x, None


def _fused_pre_map_backward(ctx, grad_out):
    x_streams, h_pre, _out = ctx.saved_tensors
    return torch.ops.flash_mhc.fused_pre_map_backward(grad_out, x_streams, h_pre)


def _fused_post_res_backward(ctx, grad_out):
    x_streams, layer_output, H_merged, h_post, _out = ctx.saved_tensors
    return torch.ops.flash_mhc.fused_post_res_backward(
        grad_out, x_streams, layer_output, H_merged, h_post)


def _mhc_coeffs_setup(ctx, inputs, output):
    proj, a_pre, a_post, a_res, bias, perm = inputs
    ctx.save_for_backward(proj, a_pre, a_post, a_res, bias, perm)


def _mhc_coeffs_backward(ctx, g_hpre, g_hpost, g_H):
    proj, a_pre, a_post, a_res, bias, perm = ctx.saved_tensors
    T = proj.shape[0]
    z = lambda *s: torch.zeros(*s, device=proj.device, dtype=torch.float32)  # noqa: E731
    g_hpre = z(T, 4) if g_hpre is None else g_hpre
    g_hpost = z(T, 4) if g_hpost is None else g_hpost
    g_H = z(T, 4, 4) if g_H is None else g_H
    g_proj, ga_pre, ga_post, ga_res, g_bias = torch.ops.flash_mhc.mhc_coeffs_backward_split(
        g_hpre, g_hpost, g_H, proj, a_pre, a_post, a_res, bias, perm)
    return g_proj, ga_pre, ga_post, ga_res, g_bias, None


torch.library.register_autograd(
    "flash_mhc::mhc_coeffs", _mhc_coeffs_backward, setup_context=_mhc_coeffs_setup)

torch.library.register_autograd(
    "flash_mhc::fused_rmsnorm_project",
    _fused_rmsnorm_project_backward,
    setup_context=_setup_save_inputs_outputs,
)
torch.library.register_autograd(
    "flash_mhc::fused_pre_map",
    _fused_pre_map_backward,
    setup_context=_setup_save_inputs_outputs,
)
torch.library.register_autograd(
    "flash_mhc::fused_post_res",
    _fused_post_res_backward,
    setup_context=_setup_save_inputs_outputs,
)
