"""CPU oracle for the mHC-lite hot path (numpy, float64 arithmetic).

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or as the timed CPU restatement.  The product
path (``flash_mhc`` and its CUDA library) never imports it and has no CPU
fallback.

This file restates, in plain numpy, the algorithm of alint77/flash-mHC for the
six fused kernels (K1/K3/K4 forward and backward), the K1 weight gradient, the
K2 coefficient math and the whole ``MHCLiteBlock`` forward/backward.  Every
function names the reference lines it follows (paths relative to the reference
project root).  Arithmetic is float64; ``bf16=True`` rounds the stored results
to bfloat16 (round-to-nearest-even) exactly where the reference kernels store a
bf16 tensor.  The restatement is pinned against tensors produced by the
reference itself (``tests/golden/make_golden.py`` and ``tests/test_oracle.py``).
"""

from __future__ import annotations

import math
from itertools import permutations

import numpy as np

# ---------------------------------------------------------------------------
# bfloat16 helpers (values are carried as float32/float64 arrays)
# ---------------------------------------------------------------------------


def bf16_round(a) -> np.ndarray:
    """Round to bfloat16 (RNE) and return float32 values.

    NaN stays NaN; overflow rounds to +-inf exactly like a hardware cvt.rn.
    """
    f = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(f)
    if nan.any():
        out[nan] = np.float32("nan")
    return out


def f32_to_bf16_bits(a) -> np.ndarray:
    """bfloat16 bit patterns (uint16) of ``a`` after RNE rounding."""
    return (bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    """float32 values of uint16 bfloat16 bit patterns."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _store(v: np.ndarray, bf16: bool) -> np.ndarray:
    return bf16_round(v) if bf16 else v.astype(np.float32)


# ---------------------------------------------------------------------------
# K1: fused RMSNorm + thin projection
# ---------------------------------------------------------------------------

K1_EPS = 1e-6  # src/flash_mhc/kernels.py:297 (rsqrt(sum_sq / nC + 1e-6))


def k1_fwd(x_flat, W, *, bf16: bool = True):
    """out[t,d] = (sum_k x[t,k] W[d,k]) * inv_rms[t]; inv_rms = rsqrt(mean x^2 + 1e-6).

    Follows src/flash_mhc/kernels.py:250-303 (project first, then scale; the
    f32 ``inv_rms`` is stored, ``out`` is stored in x's dtype).
    """
    x = np.asarray(x_flat, dtype=np.float64)
    w = np.asarray(W, dtype=np.float64)
    nC = x.shape[1]
    inv_rms = (1.0 / np.sqrt((x * x).sum(axis=1) / nC + K1_EPS)).astype(np.float32)
    acc = x @ w.T
    out = acc * inv_rms.astype(np.float64)[:, None]
    return _store(out, bf16), inv_rms


def k1_bwd_dx(grad_out, x_flat, W, proj_out, inv_rms, *, bf16: bool = True):
    """grad_x = inv_rms*(go @ W) - (sum_d go*proj) * inv_rms^2 / nC * x.

    Follows src/flash_mhc/kernels.py:306-376: the scale uses the *stored* proj
    output (not a recompute) and the f32 inv_rms.
    """
    go = np.asarray(grad_out, dtype=np.float64)
    x = np.asarray(x_flat, dtype=np.float64)
    w = np.asarray(W, dtype=np.float64)
    pr = np.asarray(proj_out, dtype=np.float64)
    r = np.asarray(inv_rms, dtype=np.float64)
    nC = x.shape[1]
    scale = (go * pr).sum(axis=1) * r * r / nC
    gx = r[:, None] * (go @ w) - scale[:, None] * x
    return _store(gx, bf16)


def k1_bwd_dw(grad_out, x_flat, inv_rms, *, bf16: bool = True):
    """grad_W = (go * inv_rms[:, None]).to(x.dtype).T @ x_flat.

    Follows src/flash_mhc/ops.py:683-684 (the scaled grad is rounded to x's dtype
    before the matmul; the matmul accumulates in f32 and stores x's dtype).
    """
    go = np.asarray(grad_out, dtype=np.float64)
    x = np.asarray(x_flat, dtype=np.float64)
    r = np.asarray(inv_rms, dtype=np.float64)
    gos = go * r[:, None]
    gos = bf16_round(gos).astype(np.float64) if bf16 else gos.astype(np.float32).astype(np.float64)
    return _store(gos.T @ x, bf16)


# ---------------------------------------------------------------------------
# K3: pre-map (4 streams -> layer input)
# ---------------------------------------------------------------------------


def k3_fwd(x_streams, h_pre, *, bf16: bool = True):
    """out[t,c] = sum_j h_pre[t,j] * x[t,j,c]  (src/flash_mhc/kernels.py:673-717)."""
    x = np.asarray(x_streams, dtype=np.float64)
    h = np.asarray(h_pre, dtype=np.float64)
    return _store(np.einsum("tj,tjc->tc", h, x), bf16)


def k3_bwd(grad_out, x_streams, h_pre, *, bf16: bool = True):
    """grad_x[t,j,c] = h_pre[t,j]*go[t,c]; grad_h[t,j] = sum_c x[t,j,c]*go[t,c].

    Follows src/flash_mhc/kernels.py:720-853 (grad_x stored in x's dtype,
    grad_h_pre in f32).
    """
    go = np.asarray(grad_out, dtype=np.float64)
    x = np.asarray(x_streams, dtype=np.float64)
    h = np.asarray(h_pre, dtype=np.float64)
    gx = h[:, :, None] * go[:, None, :]
    ghp = np.einsum("tjc,tc->tj", x, go)
    return _store(gx, bf16), ghp.astype(np.float32)


def k3_bwd_abs(grad_out, x_streams):
    """sum_c |x*go|: the scale of the f32 reductions in ``k3_bwd`` (error bounds)."""
    go = np.abs(np.asarray(grad_out, dtype=np.float64))
    x = np.abs(np.asarray(x_streams, dtype=np.float64))
    return np.einsum("tjc,tc->tj", x, go)


# ---------------------------------------------------------------------------
# K4: post-res (stream mixing + h_post-weighted layer output)
# ---------------------------------------------------------------------------


def k4_fwd(x_streams, layer_output, H_merged, h_post, *, bf16: bool = True):
    """out[t,i,c] = sum_j H[t,i,j] x[t,j,c] + h_post[t,i] lo[t,c]  (kernels.py:384-481)."""
    x = np.asarray(x_streams, dtype=np.float64)
    lo = np.asarray(layer_output, dtype=np.float64)
    H = np.asarray(H_merged, dtype=np.float64)
    hp = np.asarray(h_post, dtype=np.float64)
    out = np.einsum("tij,tjc->tic", H, x) + hp[:, :, None] * lo[:, None, :]
    return _store(out, bf16)


def k4_bwd(grad_out, x_streams, layer_output, H_merged, h_post, *, bf16: bool = True):
    """The four K4 gradients (src/flash_mhc/kernels.py:487-665).

    grad_lo[t,c]  = sum_i hp[t,i] go[t,i,c]          (x's dtype)
    grad_hp[t,i]  = sum_c go[t,i,c] lo[t,c]          (f32)
    grad_H[t,i,j] = sum_c go[t,i,c] x[t,j,c]         (f32)
    grad_x[t,j,c] = sum_i H[t,i,j] go[t,i,c]         (x's dtype)
    """
    go = np.asarray(grad_out, dtype=np.float64)
    x = np.asarray(x_streams, dtype=np.float64)
    lo = np.asarray(layer_output, dtype=np.float64)
    H = np.asarray(H_merged, dtype=np.float64)
    hp = np.asarray(h_post, dtype=np.float64)
    glo = np.einsum("ti,tic->tc", hp, go)
    ghp = np.einsum("tic,tc->ti", go, lo)
    gH = np.einsum("tic,tjc->tij", go, x)
    gx = np.einsum("tij,tic->tjc", H, go)
    return _store(gx, bf16), _store(glo, bf16), gH.astype(np.float32), ghp.astype(np.float32)


def k4_bwd_abs(grad_out, x_streams, layer_output):
    """Scales sum_c|go*lo| and sum_c|go_i*x_j| of the f32 reductions in ``k4_bwd``."""
    go = np.abs(np.asarray(grad_out, dtype=np.float64))
    x = np.abs(np.asarray(x_streams, dtype=np.float64))
    lo = np.abs(np.asarray(layer_output, dtype=np.float64))
    return np.einsum("tic,tjc->tij", go, x), np.einsum("tic,tc->ti", go, lo)


# ---------------------------------------------------------------------------
# K2: coefficient math (runs in the caller, src/flash_mhc/block.py:150-170)
# ---------------------------------------------------------------------------


def build_permutation_matrices(n: int):
    """(n!, n*n) 0/1 matrices, row i = permutation i of itertools order; identity is 0.

    Restates src/flash_mhc/block.py:21-32.
    """
    perms = list(permutations(range(n)))
    mats = np.zeros((len(perms), n * n), dtype=np.float32)
    for i, perm in enumerate(perms):
        for row, col in enumerate(perm):
            mats[i, row * n + col] = 1.0
    return mats, 0


def _sigmoid(z):
    return 1.0 / (1.0 + np.exp(-z))


def k2_coeffs(proj, alpha_pre, alpha_post, alpha_res, bias, perm, n: int = 4):
    """h_pre, h_post, H_merged from the (T, 2n+n!) projection (block.py:95-105).

    float64 throughout (the reference's f32 path); returns a dict that also
    holds the intermediates ``k2_coeffs_bwd`` needs.
    """
    p = np.asarray(proj, dtype=np.float64)
    b = np.asarray(bias, dtype=np.float64)
    P = np.asarray(perm, dtype=np.float64)
    nf = P.shape[0]
    pre, post, res = p[:, :n], p[:, n : 2 * n], p[:, 2 * n : 2 * n + nf]
    h_pre = _sigmoid(float(alpha_pre) * pre + b[:n])
    s_post = _sigmoid(float(alpha_post) * post + b[n : 2 * n])
    h_post = 2.0 * s_post
    z = float(alpha_res) * res + b[2 * n :]
    z = z - z.max(axis=1, keepdims=True)
    e = np.exp(z)
    a = e / e.sum(axis=1, keepdims=True)
    H_res = (a @ P).reshape(-1, n, n)
    H = H_res - h_post[:, :, None] * h_pre[:, None, :]
    return dict(h_pre=h_pre, h_post=h_post, H_merged=H, a=a, s_post=s_post,
                pre=pre, post=post, res=res)


def k2_coeffs_bwd(ctx, g_h_pre, g_h_post, g_H, alpha_pre, alpha_post, alpha_res, perm, n: int = 4):
    """Backward of ``k2_coeffs``: returns (g_proj, g_alpha_pre, g_alpha_post, g_alpha_res, g_bias).

    Hand-derived from the forward in src/flash_mhc/block.py:95-105 (sigmoid,
    2*sigmoid, softmax, the permutation matmul and the outer-product subtraction).
    """
    P = np.asarray(perm, dtype=np.float64)
    gH = np.asarray(g_H, dtype=np.float64)
    h_pre, h_post, a = ctx["h_pre"], ctx["h_post"], ctx["a"]
    g_hpre = np.asarray(g_h_pre, dtype=np.float64) - np.einsum("tij,ti->tj", gH, h_post)
    g_hpost = np.asarray(g_h_post, dtype=np.float64) - np.einsum("tij,tj->ti", gH, h_pre)
    ga = gH.reshape(gH.shape[0], n * n) @ P.T
    gz_res = a * (ga - (ga * a).sum(axis=1, keepdims=True))
    s = ctx["s_post"]
    gz_post = g_hpost * 2.0 * s * (1.0 - s)
    gz_pre = g_hpre * h_pre * (1.0 - h_pre)
    g_proj = np.concatenate(
        [gz_pre * float(alpha_pre), gz_post * float(alpha_post), gz_res * float(alpha_res)], axis=1
    )
    g_alpha_pre = (gz_pre * ctx["pre"]).sum()
    g_alpha_post = (gz_post * ctx["post"]).sum()
    g_alpha_res = (gz_res * ctx["res"]).sum()
    g_bias = np.concatenate([gz_pre.sum(0), gz_post.sum(0), gz_res.sum(0)])
    return g_proj, g_alpha_pre, g_alpha_post, g_alpha_res, g_bias


# ---------------------------------------------------------------------------
# Whole block (the reference's pure-PyTorch path, block.py:82-148)
# ---------------------------------------------------------------------------


def _erf(x):
    try:
        from scipy.special import erf

        return erf(x)
    except Exception:  # pragma: no cover - scipy is in the image
        return np.vectorize(math.erf)(x)


def gelu(u):
    """Exact (erf) GELU, torch.nn.functional.gelu's default."""
    return 0.5 * u * (1.0 + _erf(u / math.sqrt(2.0)))


def gelu_grad(u):
    return 0.5 * (1.0 + _erf(u / math.sqrt(2.0))) + u * np.exp(-0.5 * u * u) / math.sqrt(2.0 * math.pi)


def block_forward_backward(params: dict, x_streams, grad_out, *, rms_eps: float,
                           layer: str = "linear_gelu"):
    """Forward and backward of ``MHCLiteBlock._forward_pytorch`` in float64.

    Restates src/flash_mhc/block.py:82-148: ``F.rms_norm`` over the flattened
    n*C stream (eps = finfo(dtype).eps, passed as ``rms_eps``), normalise THEN
    project with ``W_all.weight`` (no bias inside the linear), K2, pre-map,
    the wrapped layer, post-res.  ``layer`` is ``"linear_gelu"`` (the
    reference test's ``_IdentityLinear``: gelu(x @ Wl.T), tests/test_correctness.py:320-329),
    ``"linear"`` (x @ Wl.T) or ``"identity"``.

    ``params`` keys: alpha_pre, alpha_post, alpha_res, W (D,nC), bias (D,),
    perm (n!, n*n), Wl (C,C) for the linear layers.
    Returns a dict with the forward output, intermediates and every gradient.
    """
    x = np.asarray(x_streams, dtype=np.float64)
    g = np.asarray(grad_out, dtype=np.float64)
    T, n, C = x.shape
    nC = n * C
    W = np.asarray(params["W"], dtype=np.float64)
    xf = x.reshape(T, nC)
    ms = (xf * xf).mean(axis=1)
    rinv = 1.0 / np.sqrt(ms + rms_eps)
    xn = xf * rinv[:, None]
    proj = xn @ W.T
    ap, aq, ar = params["alpha_pre"], params["alpha_post"], params["alpha_res"]
    ctx = k2_coeffs(proj, ap, aq, ar, params["bias"], params["perm"], n)
    h_pre, h_post, H = ctx["h_pre"], ctx["h_post"], ctx["H_merged"]
    li = np.einsum("tj,tjc->tc", h_pre, x)
    if layer == "identity":
        u = None
        lo = li
    else:
        Wl = np.asarray(params["Wl"], dtype=np.float64)
        u = li @ Wl.T
        lo = gelu(u) if layer == "linear_gelu" else u
    out = np.einsum("tij,tjc->tic", H, x) + h_post[:, :, None] * lo[:, None, :]

    # ---- backward ----
    g_lo = np.einsum("ti,tic->tc", h_post, g)
    g_hpost = np.einsum("tic,tc->ti", g, lo)
    g_H = np.einsum("tic,tjc->tij", g, x)
    gx = np.einsum("tij,tic->tjc", H, g)
    grads = {}
    if layer == "identity":
        g_li = g_lo
    else:
        g_u = g_lo * gelu_grad(u) if layer == "linear_gelu" else g_lo
        grads["Wl"] = g_u.T @ li
        g_li = g_u @ Wl
    gx = gx + h_pre[:, :, None] * g_li[:, None, :]
    g_hpre = np.einsum("tjc,tc->tj", x, g_li)
    g_proj, g_ap, g_aq, g_ar, g_bias = k2_coeffs_bwd(ctx, g_hpre, g_hpost, g_H, ap, aq, ar,
                                                     params["perm"], n)
    grads["W"] = g_proj.T @ xn
    g_xn = g_proj @ W
    g_xf = rinv[:, None] * g_xn - xf * ((g_xn * xf).sum(axis=1) * rinv ** 3 / nC)[:, None]
    gx = gx + g_xf.reshape(T, n, C)
    grads.update(alpha_pre=g_ap, alpha_post=g_aq, alpha_res=g_ar, bias=g_bias)
    return dict(out=out, grad_x=gx, grads=grads, h_pre=h_pre, h_post=h_post, H_merged=H,
                layer_input=li, proj=proj)


# ---------------------------------------------------------------------------
# The hot-path step that bench.py times (six kernels + the K1 weight gradient)
# ---------------------------------------------------------------------------


def hot_path_step(x_streams, W, layer_output, H_merged, h_post, h_pre,
                  g_proj, g_pre, g_post):
    """One fwd+bwd pass of K1/K3/K4 over a batch, the unit ``bench.py`` times.

    Calls the restated kernels in the order the reference's autograd runs them
    (src/flash_mhc/ops.py:678-697): K1 fwd, K3 fwd, K4 fwd, K4 bwd, K3 bwd,
    K1 bwd (grad_x and grad_W).
    """
    T, n, C = x_streams.shape
    xf = x_streams.reshape(T, n * C)
    proj, inv_rms = k1_fwd(xf, W)
    li = k3_fwd(x_streams, h_pre)
    out = k4_fwd(x_streams, layer_output, H_merged, h_post)
    g4 = k4_bwd(g_post, x_streams, layer_output, H_merged, h_post)
    g3 = k3_bwd(g_pre, x_streams, h_pre)
    gx1 = k1_bwd_dx(g_proj, xf, W, proj, inv_rms)
    gW = k1_bwd_dw(g_proj, xf, inv_rms)
    return proj, inv_rms, li, out, g4, g3, gx1, gW


def hot_path_step_f32(x_streams, W, layer_output, H_merged, h_post, h_pre,
                      g_proj, g_pre, g_post):
    """``hot_path_step`` computed in float32 with stream-unrolled numpy.

    The same restated math as the float64 functions above (same reference
    lines), written for speed so the CPU baseline in bench.py measures a
    reasonable CPU implementation, not float64 einsums.  Returns the same
    tuple as ``hot_path_step``; tests/test_oracle.py checks the two agree.
    """
    f = np.float32
    x = np.asarray(x_streams, f)
    T, n, C = x.shape
    nC = n * C
    xf = x.reshape(T, nC)
    Wf = np.asarray(W, f)
    lo = np.asarray(layer_output, f)
    H = np.asarray(H_merged, f)
    hq = np.asarray(h_post, f)
    hp = np.asarray(h_pre, f)
    # K1 fwd
    inv = (1.0 / np.sqrt(np.einsum("tk,tk->t", xf, xf) / nC + K1_EPS)).astype(f)
    proj = bf16_round((xf @ Wf.T) * inv[:, None])
    # K3 fwd
    li = hp[:, 0, None] * x[:, 0]
    for j in range(1, n):
        li += hp[:, j, None] * x[:, j]
    li = bf16_round(li)
    # K4 fwd
    out = np.empty_like(x)
    for i in range(n):
        acc = hq[:, i, None] * lo
        for j in range(n):
            acc += H[:, i, j, None] * x[:, j]
        out[:, i] = acc
    out = bf16_round(out)
    # K4 bwd
    go = np.asarray(g_post, f)
    glo = hq[:, 0, None] * go[:, 0]
    for i in range(1, n):
        glo += hq[:, i, None] * go[:, i]
    glo = bf16_round(glo)
    ghp = np.einsum("tic,tc->ti", go, lo)
    gH = np.matmul(go, x.transpose(0, 2, 1))
    gx4 = np.empty_like(x)
    for j in range(n):
        acc = H[:, 0, j, None] * go[:, 0]
        for i in range(1, n):
            acc += H[:, i, j, None] * go[:, i]
        gx4[:, j] = acc
    gx4 = bf16_round(gx4)
    # K3 bwd
    g3 = np.asarray(g_pre, f)
    gx3 = bf16_round(hp[:, :, None] * g3[:, None, :])
    gh3 = np.einsum("tjc,tc->tj", x, g3)
    # K1 bwd (dx, dW)
    gp = np.asarray(g_proj, f)
    s = np.einsum("td,td->t", gp, proj) * inv * inv / nC
    gx1 = bf16_round(inv[:, None] * (gp @ Wf) - s[:, None] * xf)
    gos = bf16_round(gp * inv[:, None])
    gW = bf16_round(gos.T @ xf)
    return proj, inv, li, out, (gx4, glo, gH, ghp), (gx3, gh3), gx1, gW
