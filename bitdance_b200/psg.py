"""Drop-in for the reference operator ``compile_preshuffle_gemm_a8`` on its W4A6-transcode path.

Reference: psg_preshuffle_gemm.py:251-277 (signature), :338-412 (in_dtype resolution),
:553-618 (split_k / split_reduce validation), :3211-3253 (launcher). Callers:
kernel/verify_w4a6.py:100-119 and kernel/bench_sweep.py:30-161.

``compile_preshuffle_gemm_a8(M=..., N=..., K=..., tile_m=..., tile_n=..., tile_k=128,
in_dtype="w4a6_tc", out_dtype="bf16", split_k=..., split_reduce=..., epilogue=...)`` returns
``launch_fn(arg_c, arg_a, arg_b, arg_scale_a, arg_scale_b, arg_bias, arg_lut, M, N, stream)``
with the reference's argument order and meaning:

* arg_c: C (M, N) in out_dtype; with split_k > 1 and split_reduce="planes" a (split_k, M, N)
  buffer of partial planes the caller sums; with "atomic" an fp32 (M, N) buffer the caller
  zeroes.
* arg_a: (M, K) u8 MXFP6 activations, arg_scale_a: E8M0 bytes, arg_b: (N, K/2) u8 NVFP4
  codes, arg_scale_b: E4M3 bytes -- the reference's bytes in this library's tiles
  (``ops.pack_activations`` / ``ops.pack_weights(..., sideband="e4m3")``), which fit the
  reference's buffer sizes ``(M*K)//32*2+4096`` and ``(N*K)//32*2+4096`` bytes. Buffers the
  reference scripts fill with constant or random bytes mean the same here.
  (``ops.w4a6_gemm`` with ``ops.pack_weights``' default layout is the faster native path: the
  packer does the weight-only part of the transcode once.)
* arg_bias: N bf16; arg_lut: accepted and ignored (the transcode tables are compiled into
  the kernel); M, N: ints; stream: a torch stream, a raw handle or None (torch's current
  stream).

``in_dtype="w4a6"`` (the reference's MXFP6 x MXFP4 arm, psg_preshuffle_gemm.py:411-423, which
kernel/verify_w4a6.py:166-172 uses as its bit-exact cross-check) takes arg_scale_b as one E8M0
byte per 32-block (N*K/32 bytes, in the block order of the E4M3 sideband); each becomes the
E4M3 byte pair of the same power of two (bd_scales_e8m0_to_e4m3_pairs), for which the NVFP4
transcode reproduces the MXFP4 block exactly, and the same GEMM runs. E8M0 exponents outside
[-9, 8] have no E4M3 form (BD_DEVERR_RANGE).

Pointers may be torch tensors, ints, or objects with ``.value`` / ``.data_ptr()``. The
per-tensor fp32 scale of the NVFP4 weights, which the reference signature has no slot for,
is the keyword ``b_tensor_scale`` (default 1.0).

Errors follow the reference: ValueError for an unknown dtype, out_dtype, split_k or
split_reduce combination; NotImplementedError for dtypes outside the W4A6 family
(w4a6_tc / w6a6_tc / w4a6) and for tile_k != 128.
"""
from __future__ import annotations

import ctypes
import functools
from typing import Optional

from . import _lib
from ._lib import call

KNOWN_DTYPES = ("fp8", "int8", "int4", "fp16", "bf16", "fp4", "fp6", "w4a6", "w6a6",
                "w6a6_tc", "w4a4_tc", "w4a6_tc")
_EPI = {"none": _lib.BD_EPI_NONE, "bias": _lib.BD_EPI_BIAS, "bias_relu": _lib.BD_EPI_BIAS_RELU,
        "bias_silu": _lib.BD_EPI_BIAS_SILU, "bias_gelu": _lib.BD_EPI_BIAS_GELU}


def _addr(x) -> Optional[int]:
    if x is None:
        return None
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    if hasattr(x, "value"):
        return int(x.value)
    return int(x)


def _stream(stream):
    # like the reference scripts (kernel/bench_sweep.py:292), None means torch's current stream
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    if hasattr(stream, "cuda_stream"):
        return ctypes.c_void_p(stream.cuda_stream)
    return ctypes.c_void_p(int(stream))


class W4A6Launcher:
    """The compiled operator: call it like the reference's launch_fn."""

    def __init__(self, K, split_k, split_reduce, out_dtype, epilogue, tiles, in_dtype="w4a6_tc"):
        self.K = K
        self.split_k = split_k
        self.split_reduce = split_reduce
        self.out_dtype = out_dtype
        self.epilogue = epilogue
        self.tiles = tiles
        self.in_dtype = in_dtype
        self._ws = {}
        self._pairs = {}   # (device, bytes) -> E4M3 scale pairs of the "w4a6" arm

    def _mxfp4_scales(self, arg_scale_b, N, stream):
        """The "w4a6" arm's E8M0 weight scales (one byte per 32-block, in the order of the
        E4M3 sideband's blocks) as E4M3 byte pairs of the same powers of two."""
        import torch
        nblk = N * self.K // 32
        dev = torch.cuda.current_device()
        key = (dev, nblk)
        if key not in self._pairs:
            self._pairs[key] = torch.empty(2 * nblk, dtype=torch.uint8, device="cuda")
        buf = self._pairs[key]
        call("bd_scales_e8m0_to_e4m3_pairs", ctypes.c_void_p(_addr(arg_scale_b)),
             ctypes.c_void_p(buf.data_ptr()), nblk, stream)
        return buf.data_ptr()

    def workspace_bytes(self, M, N):
        return 0  # planes / atomic / split_k=1 need none

    def __call__(self, arg_c, arg_a, arg_b, arg_scale_a, arg_scale_b, arg_bias, arg_lut, M, N,
                 stream=None, *, b_tensor_scale: float = 1.0):
        M, N = int(M), int(N)
        mode = _lib.BD_SPLIT_ATOMIC if self.split_reduce == "atomic" else _lib.BD_SPLIT_PLANES
        out = {"bf16": _lib.BD_OUT_BF16, "fp16": _lib.BD_OUT_F16}[self.out_dtype]
        if self.split_reduce == "atomic":
            out = _lib.BD_OUT_F32
        epi = _EPI[self.epilogue]
        bias = _addr(arg_bias) if epi != _lib.BD_EPI_NONE else None
        s = _stream(stream)
        scale_b = _addr(arg_scale_b)
        if self.in_dtype == "w4a6":
            scale_b = self._mxfp4_scales(arg_scale_b, N, s)
        call("bd_w4a6_gemm_ex", ctypes.c_void_p(_addr(arg_c)), ctypes.c_void_p(_addr(arg_a)),
             ctypes.c_void_p(_addr(arg_scale_a)), ctypes.c_void_p(_addr(arg_b)),
             ctypes.c_void_p(scale_b), float(b_tensor_scale),
             None if bias is None else ctypes.c_void_p(bias), M, N, self.K, self.split_k, mode,
             out, epi, None, 0, _lib.BD_GEMM_B_E4M3, s)


@functools.lru_cache(maxsize=1024)
def compile_preshuffle_gemm_a8(*, M: int = 0, N: int = 0, K: int, tile_m: int, tile_n: int,
                               tile_k: int, in_dtype: str = "fp8", out_dtype: str = "fp16",
                               lds_stage: int = 2, use_cshuffle_epilog: bool = False,
                               waves_per_eu: Optional[int] = None, use_async_copy: bool = False,
                               dsrd_preload: int = -1, dvmem_preload: int = -1,
                               epilogue: str = "none", xcd_swizzle: int = 0,
                               use_hw_transcode: Optional[bool] = None, split_k: int = 1,
                               split_reduce: str = "planes") -> W4A6Launcher:
    """Validate the configuration the way the reference does and return the launcher.

    The AMD-specific tuning knobs (lds_stage, waves_per_eu, use_async_copy, dsrd/dvmem
    preload, xcd_swizzle, use_cshuffle_epilog) have no meaning on sm_100a and are accepted
    for signature compatibility. use_hw_transcode=True is rejected: the hardware converts
    round ties to even and are not bit-exact to the transcode table (psg:39-49)."""
    if in_dtype not in KNOWN_DTYPES:
        raise ValueError(f"in_dtype must be one of {KNOWN_DTYPES}, got {in_dtype!r}")
    if in_dtype not in ("w4a6_tc", "w6a6_tc", "w4a6"):
        raise NotImplementedError(
            f"in_dtype={in_dtype!r} is not the W4A6 transcode path this library implements")
    if out_dtype not in ("fp16", "bf16"):
        raise ValueError(f"out_dtype must be 'fp16' or 'bf16', got {out_dtype!r}")
    if int(tile_k) != 128:
        raise NotImplementedError("w4a6_tc requires tile_k=128")
    if use_hw_transcode:
        raise NotImplementedError(
            "use_hw_transcode rounds ties to even and is not bit-exact to the transcode LUT")
    if epilogue not in _EPI:
        raise ValueError(f"unknown epilogue {epilogue!r}")
    if K % 128:
        raise ValueError(f"K={K} must be a multiple of 128")
    split_k = int(split_k)
    if split_k < 1:
        raise ValueError(f"split_k must be >= 1, got {split_k}")
    if split_k > 1:
        if K % split_k:
            raise ValueError(f"split_k={split_k} must divide K={K}")
        if (K // split_k) % int(tile_k):
            raise ValueError(f"split_k={split_k} gives a K slice of {K // split_k}, which is not "
                             f"a multiple of tile_k={tile_k}")
    if split_reduce not in ("planes", "atomic"):
        raise ValueError(f"split_reduce must be 'planes' or 'atomic', got {split_reduce!r}")
    if split_reduce == "atomic":
        if use_cshuffle_epilog:
            raise ValueError("split_reduce='atomic' requires use_cshuffle_epilog=False")
        if epilogue != "none":
            raise ValueError(f"split_reduce='atomic' cannot be combined with epilogue={epilogue!r}")
    if split_reduce == "planes" and split_k > 1 and epilogue != "none":
        raise ValueError("a bias/activation epilogue needs the full sum; use split_k=1")
    _lib.load()
    return W4A6Launcher(int(K), split_k, split_reduce, out_dtype, epilogue,
                        (int(tile_m), int(tile_n), int(tile_k)), in_dtype)
