"""``MHCLiteBlock``: the mHC-lite residual wrapper, drop-in for the reference's.

Same constructor, parameters, buffer, state_dict layout, path predicate and
activation-checkpointing semantics as src/flash_mhc/block.py:21-231 of
alint77/flash-mHC, so checkpoints and call sites move over unchanged.

Per token the block (K1) RMS-normalises the flattened n*C stream and projects
it onto 2n + n! logits, (K2) maps them to h_pre (n), h_post (n) and a
doubly-stochastic H_res (n x n) built as a convex combination of the n!
permutation matrices, (K3) pre-mixes the streams into the wrapped layer's
input, runs the layer, and (K4) post-mixes H_merged @ x + h_post * layer_out.

The fused path (CUDA + bfloat16 + (T, n, C) + n == 4) runs K1, K2, K3 and K4
as sm_100a kernels behind ``torch.ops.flash_mhc`` inside two autograd
functions that save only what the backward kernels read (x, the layer output,
the 32 projection logits, inv_rms and the f32 coefficients: ~170 bytes per
token besides x and the layer output) and recompute nothing.  Activation
checkpointing is therefore unnecessary on this path: with
``activation_checkpointing=True`` the reference re-runs K1, K2, K3 and K4 in
the backward to avoid storing layer_input and the block output; the fused path
never stores those either, so the flag leaves its memory and results unchanged
and skips the recomputation.  Every other input takes the pure-PyTorch path
(which is also what runs on CPU), with the flag honoured through torch
checkpointing exactly as in the reference.  The constructor argument keeps its
reference name ``triton_fused``; here it selects the CUDA kernels.
"""

from __future__ import annotations

import math
from itertools import permutations

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as _checkpoint

from . import ops as _ops  # noqa: F401  (registers torch.ops.flash_mhc.*)


class _StreamGrad:
    """Hands K4's share of grad_x from the post-res backward to the pre-map backward.

    The post-res backward always runs first (the pre-map's outputs feed it).
    Instead of writing K4's grad_x (sum_i H[i, j] * g_out[i]) and returning it
    to the autograd engine, which would add it to the pre-map's grad_x with a
    separate full pass, it parks K4's upstream gradient and H_merged here, and
    the pre-map backward forms K4's term inside its one combining pass: one
    (T, n, C) write and one read fewer.
    """

    __slots__ = ("g_out", "H")

    def __init__(self):
        self.g_out = None
        self.H = None


class _FusedPreMap(torch.autograd.Function):
    """K1 (RMSNorm + projection), K2 (coefficients), K3 (pre-map) forward, as
    one ``mhc_pre_forward`` call (K2 runs in K1's epilogue; at few tokens K3
    too, one launch in all).

    Backward from saved tensors only (no forward kernel is re-run):
    K3's grad_h_pre -> K2 bwd -> K1 bwd (grad_x and grad_W in one pass), then
    one pass forming grad_x = K1's + h_pre * grad_layer_input + K4's, K4's
    term computed there from the block's output gradient and H_merged.
    """

    @staticmethod
    def forward(ctx, x, W, a_pre, a_post, a_res, bias, perm, slot):
        ops = torch.ops.flash_mhc
        T, n, C = x.shape
        layer_input, proj, inv, h_pre, h_post, H = ops.mhc_pre_forward(
            x, W, a_pre, a_post, a_res, bias, perm)
        ctx.save_for_backward(x, W, proj, inv, h_pre, a_pre, a_post, a_res, bias, perm)
        ctx.slot = slot
        return layer_input, H, h_post

    @staticmethod
    def backward(ctx, g_li, g_H, g_hpost):
        ops = torch.ops.flash_mhc
        x, W, proj, inv, h_pre, a_pre, a_post, a_res, bias, perm = ctx.saved_tensors
        T, n, C = x.shape
        z = lambda *s: torch.zeros(*s, device=x.device, dtype=torch.float32)  # noqa: E731
        if g_li is None:
            g_li = torch.zeros((T, C), device=x.device, dtype=x.dtype)
        g_hpre = ops.pre_map_grad_h(g_li, x, h_pre)
        g_proj, ga_pre, ga_post, ga_res, g_bias = ops.mhc_coeffs_backward_split(
            g_hpre, z(T, 4) if g_hpost is None else g_hpost, z(T, 4, 4) if g_H is None else g_H,
            proj, a_pre, a_post, a_res, bias, perm)
        gx1, gW = ops.fused_rmsnorm_project_backward(g_proj, x.reshape(T, n * C), W, proj, inv)
        g_out, H = ctx.slot.g_out, ctx.slot.H
        ctx.slot.g_out = ctx.slot.H = None
        if g_out is None:
            gx = ops.mhc_grad_x_combine(gx1.view(T, n, C), g_li, h_pre, None)
        else:
            gx = ops.mhc_grad_x_combine_post(gx1.view(T, n, C), g_li, h_pre, g_out, H)
        return gx, gW, ga_pre, ga_post, ga_res, g_bias, None, None


class _FusedPostRes(torch.autograd.Function):
    """K4 forward; backward K4 bwd from the saved inputs (the output is not kept).

    The backward computes grad_layer_output, grad_H and grad_h_post only; K4's
    grad_x is formed by the pre-map backward from what is parked in ``slot``
    (see _StreamGrad), and the engine receives None for x from here.
    """

    @staticmethod
    def forward(ctx, x, layer_output, H_merged, h_post, slot):
        ctx.save_for_backward(x, layer_output, H_merged, h_post)
        ctx.slot = slot
        return torch.ops.flash_mhc.fused_post_res(x, layer_output, H_merged, h_post)

    @staticmethod
    def backward(ctx, g_out):
        x, lo, H, hp = ctx.saved_tensors
        g_out = g_out.contiguous()
        glo, gH, ghp = torch.ops.flash_mhc.post_res_grad_params(g_out, x, lo, H, hp)
        ctx.slot.g_out, ctx.slot.H = g_out, H
        return None, glo, gH, ghp, None


def build_permutation_matrices(n: int) -> tuple[torch.Tensor, int]:
    """All n! permutation matrices, flattened row-major to (n!, n*n), in
    itertools.permutations order; index 0 is the identity."""
    rows = []
    for perm in permutations(range(n)):
        m = torch.zeros(n, n)
        m[torch.arange(n), torch.tensor(perm)] = 1.0
        rows.append(m.reshape(-1))
    return torch.stack(rows), 0


class MHCLiteBlock(nn.Module):
    """mHC-lite wrapper around a ``(T, C) -> (T, C)`` layer with ``n_streams`` residual streams.

    forward(x_streams (T, n, C), **kwargs) -> (T, n, C); kwargs go to the layer.
    """

    def __init__(
        self,
        n_streams: int,
        hidden_size: int,
        layer: nn.Module,
        triton_fused: bool = True,
        activation_checkpointing: bool = False,
    ) -> None:
        super().__init__()
        self.n = n_streams
        self.C = hidden_size
        self.nC = n_streams * hidden_size
        self.layer = layer
        self.triton_fused = triton_fused
        self.activation_checkpointing = activation_checkpointing
        self.n_fact = math.factorial(n_streams)

        self.alpha_pre = nn.Parameter(torch.tensor([0.01]))
        self.alpha_post = nn.Parameter(torch.tensor([0.01]))
        self.alpha_res = nn.Parameter(torch.tensor([0.01]))
        self.W_all = nn.Linear(self.nC, 2 * n_streams + self.n_fact, bias=True)

        perm_flat, self.identity_idx = build_permutation_matrices(n_streams)
        self.register_buffer("perm_mat", perm_flat)

    # ------------------------------------------------------------ helpers
    def _use_activation_checkpointing(self, x_streams: torch.Tensor) -> bool:
        return (
            self.activation_checkpointing
            and self.training
            and torch.is_grad_enabled()
            and x_streams.requires_grad
        )

    def _uses_fused_path(self, x_streams: torch.Tensor) -> bool:
        return (
            self.triton_fused
            and x_streams.is_cuda
            and x_streams.dtype == torch.bfloat16
            and x_streams.dim() == 3
            and self.n == 4
        )

    def _coeffs_from_proj(self, all_proj: torch.Tensor, dt: torch.dtype):
        """K2: logits (..., 2n+n!) -> h_pre, h_post, H_merged, in dtype ``dt``."""
        n = self.n
        pre_proj, post_proj, res_proj = all_proj.split([n, n, self.n_fact], dim=-1)
        bias = self.W_all.bias.to(dt)
        h_pre = torch.sigmoid(self.alpha_pre.to(dt) * pre_proj + bias[:n])
        h_post = 2.0 * torch.sigmoid(self.alpha_post.to(dt) * post_proj + bias[n : 2 * n])
        a_res = F.softmax(self.alpha_res.to(dt) * res_proj + bias[2 * n :], dim=-1)
        H_res = torch.matmul(a_res, self.perm_mat.to(dt)).unflatten(-1, (n, n))
        H_merged = H_res - h_post.unsqueeze(-1) * h_pre.unsqueeze(-2)
        return h_pre, h_post, H_merged

    # ------------------------------------------------------- pure PyTorch
    def _mhc_coeffs_pytorch(self, x_streams: torch.Tensor):
        dt = x_streams.dtype
        x_flat = x_streams.reshape(*x_streams.shape[:-2], self.nC)
        x_norm = F.rms_norm(x_flat, (self.nC,))
        all_proj = F.linear(x_norm, self.W_all.weight.to(dt), None)
        return self._coeffs_from_proj(all_proj, dt)

    def _mhc_pre_map_pytorch(self, x_streams: torch.Tensor):
        h_pre, h_post, H_merged = self._mhc_coeffs_pytorch(x_streams)
        layer_input = torch.matmul(h_pre.unsqueeze(-2), x_streams).squeeze(-2)
        return layer_input, H_merged, h_post

    def _mhc_post_res_pytorch(self, x_streams, layer_output, H_merged, h_post):
        return (
            torch.matmul(H_merged, x_streams)
            + h_post.unsqueeze(-1) * layer_output.unsqueeze(-2)
        )

    def _run(self, x_streams, pre_map, post_res, **kwargs):
        if self._use_activation_checkpointing(x_streams):
            layer_input, H_merged, h_post = _checkpoint(pre_map, x_streams, use_reentrant=False)
            layer_output = self.layer(layer_input, **kwargs)
            return _checkpoint(post_res, x_streams, layer_output, H_merged, h_post,
                               use_reentrant=False)
        layer_input, H_merged, h_post = pre_map(x_streams)
        layer_output = self.layer(layer_input, **kwargs)
        return post_res(x_streams, layer_output, H_merged, h_post)

    def _forward_pytorch(self, x_streams: torch.Tensor, **kwargs) -> torch.Tensor:
        return self._run(x_streams, self._mhc_pre_map_pytorch, self._mhc_post_res_pytorch,
                         **kwargs)

    # ------------------------------------------------------------- fused
    def _mhc_coeffs_triton(self, x_streams: torch.Tensor):
        """K1 + K2 through the ops: f32 coefficients from the bf16 logits, with the
        parameters rounded to bf16 as the reference's ``.to(dt)`` does."""
        dt = x_streams.dtype
        T = x_streams.shape[0]
        x_flat = x_streams.reshape(T, self.nC)
        all_proj, _inv_rms = torch.ops.flash_mhc.fused_rmsnorm_project(
            x_flat, self.W_all.weight.to(dt))
        return torch.ops.flash_mhc.mhc_coeffs(all_proj, self.alpha_pre, self.alpha_post,
                                             self.alpha_res, self.W_all.bias, self.perm_mat)

    def _mhc_pre_map_triton(self, x_streams: torch.Tensor, slot=None):
        return _FusedPreMap.apply(x_streams, self.W_all.weight.to(x_streams.dtype),
                                  self.alpha_pre, self.alpha_post, self.alpha_res,
                                  self.W_all.bias, self.perm_mat,
                                  _StreamGrad() if slot is None else slot)

    def _mhc_post_res_triton(self, x_streams, layer_output, H_merged, h_post, slot=None):
        if slot is None:  # standalone use: K4's grad_x must reach the engine
            return torch.ops.flash_mhc.fused_post_res(x_streams, layer_output, H_merged, h_post)
        return _FusedPostRes.apply(x_streams, layer_output, H_merged, h_post, slot)

    def _forward_fused_no_grad(self, x_streams: torch.Tensor, **kwargs) -> torch.Tensor:
        """Inference (grad disabled, not under torch.compile): the same kernels
        called without the autograd Functions and the op dispatcher, whose host
        cost dominates at small T (~200 -> ~70 us per forward at T = 1)."""
        dt = x_streams.dtype
        W = self.W_all.weight
        if W.dtype != dt:
            W = W.to(dt)
        layer_input, _proj, _inv, _h_pre, h_post, H_merged = _ops._mhc_pre_forward_cuda(
            x_streams, W, self.alpha_pre, self.alpha_post, self.alpha_res, self.W_all.bias,
            self.perm_mat)
        layer_output = self.layer(layer_input, **kwargs)
        return _ops._fused_post_res_cuda(x_streams, layer_output, H_merged, h_post)

    def _forward_triton(self, x_streams: torch.Tensor, **kwargs) -> torch.Tensor:
        if not torch.is_grad_enabled() and not torch.compiler.is_compiling():
            return self._forward_fused_no_grad(x_streams, **kwargs)
        # No torch checkpointing here: the fused autograd functions already keep
        # only the small per-token tensors their backward kernels read.
        slot = _StreamGrad()
        layer_input, H_merged, h_post = self._mhc_pre_map_triton(x_streams, slot)
        layer_output = self.layer(layer_input, **kwargs)
        return self._mhc_post_res_triton(x_streams, layer_output, H_merged, h_post, slot)

    # The reference name is kept above; this alias says what runs.
    _forward_fused = _forward_triton

    def forward(self, x_streams: torch.Tensor, **kwargs) -> torch.Tensor:
        if self._uses_fused_path(x_streams):
            return self._forward_triton(x_streams, **kwargs)
        return self._forward_pytorch(x_streams, **kwargs)
