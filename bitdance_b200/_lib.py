"""ctypes binding of the C ABI in include/bitdance_b200.h.

The shared library is built in-tree (``bitdance_b200/libbitdance_b200.so``) by
``bitdance_b200.build.build_library()``. There is no fallback: if the library cannot be
loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libbitdance_b200.so")

BD_OK = 0
BD_ERR_INVALID_ARG = -1
BD_ERR_SHAPE = -2
BD_ERR_ALIGNMENT = -3
BD_ERR_ARCH = -4
BD_ERR_CUDA = -5
BD_ERR_WORKSPACE = -6
BD_ERR_DEVICE = -7

BD_OUT_BF16, BD_OUT_F16, BD_OUT_F32 = 0, 1, 2
BD_EPI_NONE, BD_EPI_BIAS, BD_EPI_BIAS_RELU, BD_EPI_BIAS_SILU, BD_EPI_BIAS_GELU = 0, 1, 2, 3, 4
BD_SPLIT_REDUCE, BD_SPLIT_PLANES, BD_SPLIT_ATOMIC = 0, 1, 2
BD_GEMM_OVERLAP_PREV, BD_GEMM_WEIGHTS_STATIC, BD_GEMM_B_E4M3, BD_GEMM_SINGLE_CTA = 1, 2, 4, 8
BD_IN_F32, BD_IN_BF16 = 0, 1
BD_DEVERR_WAIT_MASK, BD_DEVERR_WAIT_TMA, BD_DEVERR_NONFINITE, BD_DEVERR_RANGE = 0x1F, 0x01, 0x20, 0x40

# name -> (restype, argtypes); mirrors include/bitdance_b200.h
_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_F = ctypes.c_float
SIGNATURES = {
    "bd_version": (_I, []),
    "bd_status_string": (ctypes.c_char_p, [_I]),
    "bd_device_error": (_I, [ctypes.POINTER(ctypes.c_uint32), _I]),
    "bd_selftest_bounded_wait": (_I, [_I64, _P]),
    "bd_probe_mma_peak": (_I, [_I64, _I, _I, _P]),
    "bd_transcode_nvfp4_to_mxfp6": (_I, [_P, _P, _P, _P, _I64, _I, _P]),
    "bd_pack_b": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "bd_pack_b_e4m3": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "bd_pack_a": (_I, [_P, _P, _P, _P, _I, _I, _P]),
    "bd_scales_e8m0_to_e4m3_pairs": (_I, [_P, _P, _I64, _P]),
    "bd_quantize_a_mxfp6": (_I, [_P, _I, _P, _P, _P, _I, _I, _P]),
    "bd_quantize_b_nvfp4": (_I, [_P, _I, _P, _P, _P, _I, _I, _P]),
    "bd_quantize_a_mxfp6_ex": (_I, [_P, _I, _P, _P, _P, _I, _I, ctypes.c_uint, _P]),
    "bd_query_workspace": (_SZ, [_I, _I, _I, _I, _I]),
    "bd_w4a6_gemm": (_I, [_P, _P, _P, _P, _P, _F, _P, _I, _I, _I, _I, _I, _I, _I, _P, _SZ, _P]),
    "bd_w4a6_gemm_ex": (_I, [_P, _P, _P, _P, _P, _F, _P, _I, _I, _I, _I, _I, _I, _I, _P, _SZ,
                             ctypes.c_uint, _P]),
    "bd_w4a6_gemm_noalloc": (_I, [_P, _P, _P, _P, _P, _F, _P, _I, _I, _I, _I, _I, _P]),
    "bd_splitk_reduce": (_I, [_P, _P, _P, _F, _I, _I, _I, _I, _I, _P]),
}


class BitdanceError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int, text: str):
        super().__init__(f"{fn} failed: status {status} ({text})")
        self.status = status


_lib = None
_lock = threading.Lock()


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library. Raises OSError if it is missing."""
    global _lib
    with _lock:
        if _lib is None:
            p = path or LIB_PATH
            if not os.path.exists(p):
                raise OSError(
                    f"{p} not found: build it with `python -c 'import __graft_entry__ as g; g.build()'`"
                    " (the CUDA extension is required; there is no CPU fallback)")
            lib = ctypes.CDLL(p)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


def status_text(status: int) -> str:
    return load().bd_status_string(int(status)).decode()


def check(fn: str, status: int) -> None:
    if status != BD_OK:
        raise BitdanceError(fn, status, status_text(status))


def call(fn: str, *args) -> int:
    """Call an int-returning entry point and raise BitdanceError on a non-zero status."""
    st = getattr(load(), fn)(*args)
    check(fn, st)
    return st
