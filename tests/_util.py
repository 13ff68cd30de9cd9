"""Helpers shared by the test files (loading fixtures, tolerance checks)."""

from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_golden(name: str) -> dict:
    """Load ``tests/golden/<name>.npz``; uint16 arrays are bf16 bit patterns -> float32."""
    from oracle.mhc_oracle import bf16_bits_to_f32

    z = np.load(GOLDEN / f"{name}.npz")
    out = {}
    for k in z.files:
        a = z[k]
        out[k] = bf16_bits_to_f32(a) if a.dtype == np.uint16 else a
        if a.dtype == np.uint16:
            out[k + "__bf16"] = True
    return out


def assert_close(name, actual, expected, atol, rtol):
    """allclose with a max-abs / max-rel report (the reference's own helper,
    tests/test_correctness.py:67-78, restated)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, f"{name}: shape {a.shape} vs {e.shape}"
    diff = np.abs(a - e)
    ok = bool(np.all(diff <= atol + rtol * np.abs(e)))
    if not ok:
        rel = diff / np.maximum(np.abs(e), 1e-8)
        i = int(np.argmax(diff - (atol + rtol * np.abs(e))))
        raise AssertionError(
            f"{name}: max_abs={diff.max():.4e} max_rel={rel.max():.4e} "
            f"(atol={atol}, rtol={rtol}); worst idx {np.unravel_index(i, a.shape)} "
            f"actual={a.flat[i]!r} expected={e.flat[i]!r}")


def assert_sum_close(name, actual, expected, abs_scale, rel):
    """|actual - expected| <= rel * abs_scale elementwise.

    For f32 reductions (sum_c a*b) the rounding error is bounded by a multiple
    of sum_c |a*b| (``abs_scale``), not of |result|, because terms cancel.
    """
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    s = np.asarray(abs_scale, dtype=np.float64)
    assert a.shape == e.shape == s.shape, f"{name}: shapes {a.shape} {e.shape} {s.shape}"
    diff = np.abs(a - e)
    lim = rel * s + 1e-30
    if not np.all(diff <= lim):
        i = int(np.argmax(diff / lim))
        raise AssertionError(
            f"{name}: worst |diff|/bound={diff.flat[i] / lim.flat[i]:.3g} at "
            f"{np.unravel_index(i, a.shape)} actual={a.flat[i]!r} expected={e.flat[i]!r} "
            f"scale={s.flat[i]!r} (rel={rel})")
