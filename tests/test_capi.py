"""C-ABI checks that need no GPU: the library loads, exports exactly what
include/flashmhc.h declares, and rejects bad arguments before any launch."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from flash_mhc import _native

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "flashmhc.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"FMHC_API\s+[\w\s\*]+?\b(fmhc_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    for must in ("fmhc_k1_fwd", "fmhc_k1_bwd_dx", "fmhc_k1_bwd", "fmhc_k3_fwd",
                 "fmhc_k3_bwd", "fmhc_k4_fwd", "fmhc_k4_bwd", "fmhc_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    path = _native.library_path()
    assert path.exists(), f"build the library first: make -C flash-mhc_b200 ({path})"
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted({ln.split()[-1] for ln in out.splitlines() if " T " in ln})
    assert exported == _declared()
    L = _native.lib()
    for name in _declared():
        assert hasattr(L, name)
    assert _native.version().startswith("flashmhc-sm100")


def _status(name, *args):
    L = _native.lib()
    return getattr(L, name)(*args), L.fmhc_last_error().decode()


def test_argument_validation_without_gpu():
    p = ctypes.c_void_p(16)  # never dereferenced: every case fails validation first
    st, msg = _status("fmhc_k3_fwd", p, p, p, 8, 3, 64, None)
    assert st == 1 and "n=4" in msg
    st, msg = _status("fmhc_k4_bwd", p, p, p, p, p, p, p, p, p, -1, 4, 64, None)
    assert st == 1 and "T must be" in msg
    st, msg = _status("fmhc_k1_fwd", p, p, p, p, 8, 256, 33, None)
    assert st == 2 and "D" in msg
    st, msg = _status("fmhc_k3_fwd", None, p, p, 8, 4, 64, None)
    assert st == 1 and "NULL" in msg
    st, msg = _status("fmhc_k4_fwd", p, p, ctypes.c_void_p(20), p, p, 8, 4, 64, None)
    assert st == 3 and "16-byte" in msg
    ws = ctypes.c_void_p(4096)
    st, msg = _status("fmhc_k1_bwd", p, p, p, p, p, p, p, ws, 0, 8, 256, 32, None)
    assert st == 6 and "workspace" in msg
    st, msg = _status("fmhc_k2_fwd_typed", p, p, p, p, p, 7, p, 0, p, p, p, 8, None)
    assert st == 2 and "dtype" in msg
    st, msg = _status("fmhc_mhc_grad_x_combine_post", p, p, p, p, p, p, 8, 3, 64, None)
    assert st == 1 and "n=4" in msg
    # the pre-block entry (K1 + K2 + K3): n, dtype, NULL and alignment checks
    pre = lambda **kw: _status("fmhc_mhc_pre_fwd", *[kw.get(k, d) for k, d in (  # noqa: E731
        ("x", p), ("W", p), ("a_pre", p), ("a_post", p), ("a_res", p), ("bias", p), ("pdt", 0),
        ("perm", p), ("qdt", 0), ("proj", p), ("inv", p), ("h_pre", p), ("h_post", p), ("H", p),
        ("li", p), ("T", 8), ("n", 4), ("C", 64), ("stream", None))])
    st, msg = pre(n=3)
    assert st == 1 and "n=4" in msg
    st, msg = pre(pdt=5)
    assert st == 2 and "dtype" in msg
    st, msg = pre(proj=None)
    assert st == 1 and "NULL" in msg
    st, msg = pre(h_pre=ctypes.c_void_p(20))
    assert st == 3 and "16-byte" in msg
    st, msg = pre(x=None, W=None, proj=None, T=0)
    assert st == 0 and msg == ""
    # K4 backward accepts grad_x = NULL (parameter gradients only); the other
    # outputs are still required
    st, msg = _status("fmhc_k4_bwd", p, p, p, p, p, None, None, p, p, 8, 4, 64, None)
    assert st == 1 and "NULL" in msg
    # T == 0 is a no-op that succeeds without touching the device
    st, msg = _status("fmhc_k4_bwd", None, None, None, None, None, None, None, None, None,
                      0, 4, 64, None)
    assert st == 0 and msg == ""


def test_python_raises_value_error_for_invalid_argument():
    with pytest.raises(ValueError):
        _native.call("fmhc_k3_fwd", ctypes.c_void_p(16), ctypes.c_void_p(16),
                     ctypes.c_void_p(16), 8, 5, 64, None)


def test_workspace_size_query():
    assert _native.workspace_size_k1_bwd(0, 4096, 32) == 0
    n = _native.workspace_size_k1_bwd(65536, 4096, 32)
    assert n > 0 and n % 256 == 0
