"""Shared test set-up: the `gpu` marker, import paths and the CPU checker library."""
import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="session")
def orc():
    """The C restatement of the transcode (oracle/liborc.so), built on demand."""
    lib_path = os.path.join(ROOT, "oracle", "liborc.so")
    src = os.path.join(ROOT, "oracle", "w4a6_ref.c")
    if not os.path.exists(lib_path) or os.path.getmtime(lib_path) < os.path.getmtime(src):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True,
                       capture_output=True)
    lib = ctypes.CDLL(lib_path)
    lib.orc_transcode.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int,
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    lib.orc_dequant.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                ctypes.c_void_p, ctypes.c_int]
    lib.orc_tables.argtypes = [ctypes.c_void_p] * 3
    return lib


def orc_transcode(lib, codes_packed, scales, scale_block=16, nthreads=4):
    codes_packed = np.ascontiguousarray(codes_packed, np.uint8).reshape(-1)
    scales = np.ascontiguousarray(scales, np.uint8).reshape(-1)
    nb = codes_packed.size // 16
    e6 = np.empty(nb * 32, np.uint8)
    e8 = np.empty(nb, np.uint8)
    rc = lib.orc_transcode(codes_packed.ctypes.data, scales.ctypes.data, nb, scale_block,
                           e6.ctypes.data, e8.ctypes.data, nthreads)
    assert rc == 0
    return e6, e8


def has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
