"""Seeded inputs of the bf16-grid block fixtures (numpy only).

``make_golden.py`` feeds these to the reference's float32 pure-PyTorch block
and the GPU tests feed the same arrays to the fused bf16 block, so the two
paths see identical values: every input and parameter is a bfloat16 value
(held as float64), and numpy's PCG64 streams are reproducible across machines.

Distributions follow BASELINE configs[0] / the block configs: x and the
upstream gradient ~N(0,1); ``W_all`` weight and bias ~U(+-1/sqrt(nC)) (the
distribution of torch's default ``nn.Linear`` init); the wrapped layer's
weight ~N(0, wl_std).
"""

from __future__ import annotations

import numpy as np

from oracle.mhc_oracle import bf16_round


def _bf(a) -> np.ndarray:
    return bf16_round(a).astype(np.float64)


def block_case_inputs(T: int, C: int, seed: int, wl_std: float, alphas=(0.01, 0.01, 0.01)):
    """x (T,4,C), g (T,4,C), W (32,4C), bias (32,), Wl (C,C), alphas (3,), all bf16 values."""
    rng = np.random.default_rng(seed)
    nC = 4 * C
    x = _bf(rng.standard_normal((T, 4, C)))
    g = _bf(rng.standard_normal((T, 4, C)))
    W = _bf(rng.uniform(-1.0, 1.0, (32, nC)) / np.sqrt(nC))
    bias = _bf(rng.uniform(-1.0, 1.0, 32) / np.sqrt(nC))
    Wl = _bf(rng.standard_normal((C, C)) * wl_std)
    al = _bf(np.asarray(alphas, dtype=np.float32))
    return dict(x=x, g=g, W=W, bias=bias, Wl=Wl, alphas=al)


# name -> (T, C, seed, wl_std, alphas, gelu layer, number of tokens stored)
CASES = {
    # T=4096, C=1024, default init, Linear(1024, 1024, bias=False) ~N(0,0.02)
    "block_cfg0_fp32": (4096, 1024, 0, 0.02, (0.01, 0.01, 0.01), False, 16),
    # a small stress case: alphas moved off their init so K2's nonlinearities
    # matter, a larger layer weight and the reference test's gelu layer
    "block_grid_fp32": (48, 32, 3, 0.16, (0.7, 0.9, 1.3), True, 48),
}


def stored_rows(T: int, n_rows: int) -> np.ndarray:
    """The token rows whose per-token outputs a fixture stores (sorted)."""
    if n_rows >= T:
        return np.arange(T)
    return np.sort(np.random.default_rng(T + n_rows).choice(T, n_rows, replace=False))
