"""ctypes binding of ``libtda_b200.so`` (the C ABI declared in include/tda_b200.h).

The library is built in-tree by ``python -m tda_b200.build``.  There is no CPU
or Triton fallback: if the library is missing, every op raises.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libtda_b200.so")

TDA_F32 = 0
TDA_BF16 = 1
TDA_F16 = 2

TDA_OK = 0
TDA_ERR_INVALID = -1
TDA_ERR_UNSUPPORTED = -2
TDA_ERR_CUDA = -3
TDA_ERR_WORKSPACE = -4

# every symbol include/tda_b200.h declares, with its ctypes signature
_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_SZ = ctypes.c_size_t
SIGNATURES = {
    "tda_version": (_I, []),
    "tda_last_error": (ctypes.c_char_p, []),
    "tda_workspace_size": (_SZ, [_I, _I, _I64, _I64, _I64, _I]),
    "tda_rect_fwd": (_I, [_P, _P, _P, _P, _I, _I, _I64, _I64, _I64, _F, _F, _I, _P, _SZ, _P, _P]),
    "tda_diff_fwd": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I64, _I64, _I64, _F, _F, _F, _I, _P, _SZ, _P, _P]),
    "tda_key_inv_norms": (_I, [_P, _I, _I64, _I64, _I64, _P, _P]),
    "tda_key_inv_norms_pair": (_I, [_P, _P, _I, _I64, _I64, _I64, _P, _P, _P]),
    "tda_rect_fwd_tc": (_I, [_P, _P, _P, _P, _I, _I64, _I64, _I64, _F, _F, _I, _P, _P, _P]),
    "tda_diff_fwd_tc": (_I, [_P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _F, _F, _F, _I, _P, _P, _P, _P]),
    "tda_debug_set": (_I, [_I, ctypes.c_uint64]),
    "tda_debug_stats": (_I, [_P]),
    "tda_diff_fwd_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I64, _I64, _I64, _F, _F, _F, _I, _P, _P]),
    "tda_rect_fwd_strided": (_I, [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _F, _F, _I, _P, _SZ, _P, _P]),
    "tda_diff_fwd_strided": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I64, _F, _F, _F, _I, _P, _SZ,
                                  _P, _P]),
    "tda_diff_fwd_lambda": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I64, _I64, _I64, _I64, _F, _P, _I64, _I64, _F,
                                 _I, _P, _SZ, _P, _P]),
    "tda_bwd_workspace_size": (_SZ, [_I, _I64, _I64, _I64, _I]),
    "tda_rect_bwd": (_I, [_P, _P, _P, _P, _I, _P, _P, _P, _I64, _I64, _I64, _F, _F, _I, _F, _I, _P, _SZ, _P, _P]),
}

_lib = None


class TdaError(RuntimeError):
    """Raised when a tda_b200 C entry point returns an error code."""


def load() -> ctypes.CDLL:
    """Load the CUDA library (once) and attach signatures.  Raises if it has
    not been built: the ops never fall back to another implementation."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"tda_b200 CUDA library not found at {LIB_PATH}; build it with `python -m tda_b200.build`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != TDA_OK:
        msg = load().tda_last_error().decode(errors="replace")
        if rc in (TDA_ERR_INVALID, TDA_ERR_UNSUPPORTED, TDA_ERR_WORKSPACE):
            raise ValueError(f"tda_b200: {msg} (code {rc})")
        raise TdaError(f"tda_b200: {msg} (code {rc})")
