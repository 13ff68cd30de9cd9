"""``MHCLiteBlock``: the mHC-lite residual wrapper, drop-in for the reference's.

Same constructor, parameters, buffer, state_dict layout, path predicate and
activation-checkpointing semantics as src/flash_mhc/block.py:21-231 of
alint77/flash-mHC, so checkpoints and call sites move over unchanged.

Per token the block (K1) RMS-normalises the flattened n*C stream and projects
it onto 2n + n! logits, (K2) maps them to h_pre (n), h_post (n) and a
doubly-stochastic H_res (n x n) built as a convex combination of the n!
permutation matrices, (K3) pre-mixes the streams into the wrapped layer's
input, runs the layer, and (K4) post-mixes H_merged @ x + h_post * layer_out.

The fused path (CUDA + bfloat16 + (T, n, C) + n == 4) runs K1, K3 and K4 as
the sm_100a kernels behind ``torch.ops.flash_mhc``; K2 stays in eager torch in
the input dtype, as in the reference.  Every other input takes the
pure-PyTorch path (which is also what runs on CPU).  The constructor argument
keeps its reference name ``triton_fused``; here it selects the CUDA kernels.
"""

from __future__ import annotations

import math
from itertools import permutations

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as _checkpoint

from . import ops as _ops  # noqa: F401  (registers torch.ops.flash_mhc.*)


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
        dt = x_streams.dtype
        T = x_streams.shape[0]
        x_flat = x_streams.reshape(T, self.nC)
        all_proj, _inv_rms = torch.ops.flash_mhc.fused_rmsnorm_project(
            x_flat, self.W_all.weight.to(dt))
        return self._coeffs_from_proj(all_proj, dt)

    def _mhc_pre_map_triton(self, x_streams: torch.Tensor):
        h_pre, h_post, H_merged = self._mhc_coeffs_triton(x_streams)
        layer_input = torch.ops.flash_mhc.fused_pre_map(x_streams, h_pre.float())
        return layer_input, H_merged.float(), h_post.float()

    def _mhc_post_res_triton(self, x_streams, layer_output, H_merged, h_post):
        return torch.ops.flash_mhc.fused_post_res(x_streams, layer_output, H_merged, h_post)

    def _forward_triton(self, x_streams: torch.Tensor, **kwargs) -> torch.Tensor:
        return self._run(x_streams, self._mhc_pre_map_triton, self._mhc_post_res_triton,
                         **kwargs)

    # The reference name is kept above; this alias says what runs.
    _forward_fused = _forward_triton

    def forward(self, x_streams: torch.Tensor, **kwargs) -> torch.Tensor:
        if self._uses_fused_path(x_streams):
            return self._forward_triton(x_streams, **kwargs)
        return self._forward_pytorch(x_streams, **kwargs)
