"""ctypes binding of libflashmhc_sm100.so (the C ABI declared in include/flashmhc.h).

The library is built in-tree (``make -C flash-mhc_b200``) next to this file.
Loading is lazy: importing ``flash_mhc`` works without it (fake tensors,
the pure-PyTorch block path on CPU), but every CUDA op raises a RuntimeError
if the library is missing -- there is no silent fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_NAME = "libflashmhc_sm100.so"
_LIB_PATH = Path(os.environ.get("FLASH_MHC_LIB", Path(__file__).with_name(LIB_NAME)))

_lock = threading.Lock()
_lib = None

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64

# name -> argtypes (restype int unless listed in _RESTYPES)
_SIGNATURES = {
    "fmhc_last_error": [],
    "fmhc_version": [],
    "fmhc_check_device_error": [ctypes.POINTER(ctypes.c_int)],
    "fmhc_k1_fwd": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "fmhc_debug_k1_fwd_lost_copy": [_vp, _vp, _vp, _vp, _i64, _i64, _vp],
    "fmhc_k1_bwd_dx": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "fmhc_k1_bwd_workspace_size": [_i64, _i64, _i64],
    "fmhc_k1_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp],
    "fmhc_k2_fwd": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _vp],
    "fmhc_k2_fwd_typed": [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp, _vp, _vp,
                          _i64, _vp],
    "fmhc_k2_bwd_typed": [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp, _vp, _vp,
                          _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp],
    "fmhc_mhc_pre_fwd": [_vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp, _vp,
                         _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "fmhc_k2_bwd_workspace_size": [_i64],
    "fmhc_k2_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp],
    "fmhc_k3_fwd": [_vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "fmhc_k3_bwd": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "fmhc_mhc_grad_x_combine": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "fmhc_mhc_grad_x_combine_post": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "fmhc_k4_fwd": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "fmhc_k4_bwd": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
}
_RESTYPES = {
    "fmhc_last_error": ctypes.c_char_p,
    "fmhc_version": ctypes.c_char_p,
    "fmhc_k1_bwd_workspace_size": _i64,
    "fmhc_k2_bwd_workspace_size": _i64,
}

STATUS = {
    0: "FMHC_OK",
    1: "FMHC_ERR_INVALID_ARGUMENT",
    2: "FMHC_ERR_UNSUPPORTED",
    3: "FMHC_ERR_ALIGNMENT",
    4: "FMHC_ERR_LAUNCH",
    5: "FMHC_ERR_CUDA",
    6: "FMHC_ERR_WORKSPACE",
}


def library_path() -> Path:
    return _LIB_PATH


def lib():
    """The loaded library (raises RuntimeError if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise RuntimeError(
                    f"flash_mhc: CUDA library {_LIB_PATH} not found; build it with "
                    "`make -C flash-mhc_b200` (or __graft_entry__.build()). "
                    "There is no non-CUDA implementation of the fused ops.")
            handle = ctypes.CDLL(str(_LIB_PATH))
            for name, args in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = handle
    return _lib


class FlashMHCError(RuntimeError):
    """A C-ABI call returned a non-zero fmhc_status."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed with {STATUS.get(status, status)}: {message}")
        self.status = status


def call(name: str, *args) -> None:
    """Call C-ABI function ``name``; raise FlashMHCError on a non-zero status."""
    L = lib()
    st = getattr(L, name)(*args)
    if st != 0:
        msg = L.fmhc_last_error().decode(errors="replace")
        if st == 1:  # invalid argument: surface as ValueError like the reference
            raise ValueError(f"{name}: {msg}")
        raise FlashMHCError(name, st, msg)


def workspace_size_k1_bwd(T: int, nC: int, D: int) -> int:
    """Bytes of scratch fmhc_k1_bwd needs on the current device."""
    return int(lib().fmhc_k1_bwd_workspace_size(T, nC, D))


def check_device_error() -> int:
    """Synchronise the current device and return (and clear) its device error word."""
    code = ctypes.c_int(0)
    call("fmhc_check_device_error", ctypes.byref(code))
    return code.value


def version() -> str:
    return lib().fmhc_version().decode()
