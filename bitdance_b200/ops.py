"""Tensor-level entry points over the C ABI (device buffers are torch CUDA tensors).

PyTorch only provides device memory and the current stream here; every computation runs
in the library's own CUDA kernels.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import call

_OUT = {torch.bfloat16: _lib.BD_OUT_BF16, torch.float16: _lib.BD_OUT_F16,
        torch.float32: _lib.BD_OUT_F32}
EPILOGUES = {"none": _lib.BD_EPI_NONE, "bias": _lib.BD_EPI_BIAS,
             "bias_relu": _lib.BD_EPI_BIAS_RELU, "bias_silu": _lib.BD_EPI_BIAS_SILU,
             "bias_gelu": _lib.BD_EPI_BIAS_GELU}
SPLIT_MODES = {"reduce": _lib.BD_SPLIT_REDUCE, "planes": _lib.BD_SPLIT_PLANES,
               "atomic": _lib.BD_SPLIT_ATOMIC}


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    if stream is None:
        stream = torch.cuda.current_stream()
    s = stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
    return ctypes.c_void_p(s)


def _check_device(t, what: str):
    """The C ABI launches on the CURRENT device and builds its tensor maps, error word and
    static scratch for it: a tensor on another device would be read through the wrong
    context (an illegal-address fault) -- refuse it before the call."""
    cur = torch.cuda.current_device()
    idx = t.device.index if t.device.index is not None else cur
    if idx != cur:
        raise ValueError(f"{what} is on cuda:{idx} but the current device is cuda:{cur}; "
                         "call inside `with torch.cuda.device(...)`")


def _need(t: torch.Tensor, dtype, what: str, numel: Optional[int] = None):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{what} must be a CUDA tensor")
    _check_device(t, what)
    if t.dtype != dtype:
        raise TypeError(f"{what} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{what} must be contiguous")
    if numel is not None and t.numel() < numel:
        raise ValueError(f"{what} holds {t.numel()} elements, needs {numel}")


def transcode(codes: torch.Tensor, scales: torch.Tensor, scale_block: int = 16,
              e2m3: Optional[torch.Tensor] = None, e8m0: Optional[torch.Tensor] = None,
              stream=None):
    """NVFP4 -> MXFP6 (natural layouts). codes: packed nibbles (nblk*16 bytes); scales: E4M3
    (nblk*2 bytes for scale_block 16, nblk for 32). Returns (e2m3 codes, e8m0)."""
    if codes.numel() % 16:
        raise ValueError("codes must hold a whole number of 32-element blocks (16 bytes each)")
    nblk = codes.numel() // 16
    _need(codes, torch.uint8, "codes")
    _need(scales, torch.uint8, "scales", nblk * (2 if scale_block == 16 else 1))
    if e2m3 is None:
        e2m3 = torch.empty(nblk * 32, dtype=torch.uint8, device=codes.device)
    if e8m0 is None:
        e8m0 = torch.empty(nblk, dtype=torch.uint8, device=codes.device)
    _need(e2m3, torch.uint8, "e2m3", nblk * 32)
    _need(e8m0, torch.uint8, "e8m0", nblk)
    call("bd_transcode_nvfp4_to_mxfp6", _p(codes), _p(scales), _p(e2m3), _p(e8m0), nblk,
         scale_block, _stream(stream))
    return e2m3, e8m0


@dataclass
class PackedWeights:
    """NVFP4 weights in the GEMM's tiled, transcode-ready layout (bd_pack_b): E2M1 codes with
    their sign bits placed for the on-chip transcode, one 16-bit class word per 32-block made
    from its two E4M3 scale bytes, and the fp32 tensor scale."""
    codes: torch.Tensor    # [N/128][K/128][128][64] u8 (flat)
    scales: torch.Tensor   # [N/128][K/128][128][8]  u8 (flat): 4 class words per row and chunk
    tensor_scale: float
    N: int
    K: int
    # "class": bd_pack_b's transcode-ready layout; "e4m3": the natural codes and E4M3 scale bytes
    # only regrouped (bd_pack_b_e4m3), read with BD_GEMM_B_E4M3
    sideband: str = "class"


@dataclass
class PackedActivations:
    """MXFP6 activations in the GEMM operand layout."""
    codes: torch.Tensor    # (M, K) u8, one E2M3 code per byte (bits 0..5)
    scales: torch.Tensor   # [K/128][Mp4][4] E8M0 (flat)
    M: int
    K: int


def pack_weights(codes: torch.Tensor, scales16: torch.Tensor, tensor_scale: float = 1.0,
                 stream=None, sideband: str = "class") -> PackedWeights:
    """codes (N, K/2) packed nibbles, scales16 (N, K/16) E4M3 -> PackedWeights. sideband
    "class" (default): the transcode-ready layout; "e4m3": the reference's bytes regrouped."""
    if sideband not in ("class", "e4m3"):
        raise ValueError(f"unknown sideband {sideband!r}")
    N, Kh = codes.shape
    K = Kh * 2
    _need(codes, torch.uint8, "codes")
    _need(scales16, torch.uint8, "scales16", N * K // 16)
    tc = torch.empty(N * K // 2, dtype=torch.uint8, device=codes.device)
    ts = torch.empty(N * K // 16, dtype=torch.uint8, device=codes.device)
    call("bd_pack_b" if sideband == "class" else "bd_pack_b_e4m3", _p(codes), _p(scales16),
         _p(tc), _p(ts), N, K, _stream(stream))
    return PackedWeights(tc, ts, float(tensor_scale), N, K, sideband)


def pack_activations(codes: torch.Tensor, e8m0: torch.Tensor, stream=None,
                     inplace: bool = False) -> PackedActivations:
    """codes (M, K) one E2M3 code per byte, e8m0 (M, K/32) -> PackedActivations. The codes are
    already the operand layout; inplace=True uses `codes` itself as the operand (no copy, only
    the scales are re-laid out), so later writes to `codes` change the operand."""
    M, K = codes.shape
    _need(codes, torch.uint8, "codes")
    _need(e8m0, torch.uint8, "e8m0", M * K // 32)
    mp4 = (M + 3) // 4 * 4
    out = codes if inplace else torch.empty((M, K), dtype=torch.uint8, device=codes.device)
    sc = torch.empty((K // 32) * mp4, dtype=torch.uint8, device=codes.device)
    call("bd_pack_a", _p(codes), _p(e8m0), _p(out), _p(sc), M, K, _stream(stream))
    return PackedActivations(out, sc, M, K)


_IN = {torch.float32: _lib.BD_IN_F32, torch.bfloat16: _lib.BD_IN_BF16}


def _check_x(x: torch.Tensor, k_mult: int):
    if x.dim() != 2:
        raise ValueError("x must be 2-D (M, K)")
    if x.dtype not in _IN:
        raise TypeError(f"x must be float32 or bfloat16, got {x.dtype}")
    _need(x, x.dtype, "x")
    M, K = x.shape
    if K % k_mult:
        raise ValueError(f"K must be a multiple of {k_mult}, got {K}")
    return M, K


def quantize_mxfp6(x: torch.Tensor, stream=None):
    """Activations x (M, K) fp32/bf16 -> (E2M3 codes (M, K) u8, E8M0 (M, K/32) u8), the
    reference's Direct-MXFP6 quantize(x, E8M0, E2M3) (vector_quant_error.py:305, :389) on the
    GPU. NaN / Inf input sets BD_DEVERR_NONFINITE in the device error word (device_error())."""
    M, K = _check_x(x, 32)
    codes = torch.empty((M, K), dtype=torch.uint8, device=x.device)
    e8m0 = torch.empty((M, K // 32), dtype=torch.uint8, device=x.device)
    call("bd_quantize_a_mxfp6", _p(x), _IN[x.dtype], _p(codes), _p(e8m0), None, M, K,
         _stream(stream))
    return codes, e8m0


def quantize_activations(x: torch.Tensor, stream=None,
                         overlap_prev: bool = False) -> PackedActivations:
    """Activations x (M, K) fp32/bf16 -> PackedActivations in one launch: the quantiser writes
    the codes (already the GEMM's layout) and the tiled E8M0 scales directly. K % 128 == 0.
    overlap_prev: launched with programmatic serialisation (it waits for the previous kernel
    on the stream before reading x or writing its outputs)."""
    M, K = _check_x(x, 128)
    mp4 = (M + 3) // 4 * 4
    codes = torch.empty((M, K), dtype=torch.uint8, device=x.device)
    sc = torch.empty((K // 32) * mp4, dtype=torch.uint8, device=x.device)
    call("bd_quantize_a_mxfp6_ex", _p(x), _IN[x.dtype], _p(codes), None, _p(sc), M, K,
         _lib.BD_GEMM_OVERLAP_PREV if overlap_prev else 0, _stream(stream))
    return PackedActivations(codes, sc, M, K)


def quantize_nvfp4(w: torch.Tensor, stream=None):
    """Weights w (N, K) fp32/bf16 on the GPU -> (codes (N, K/2) packed E2M1 nibbles,
    scales16 (N, K/16) E4M3 bytes, tstat (2,) int32 device tensor: tstat[0] the fp32 tensor
    scale's bits, tstat[1] the bits of amax(|w|)): the reference's two-level NVFP4 encode
    (remote/quant_real_weights.py:273-287 + kernel/nvfp4_codec.py:34-63) on the GPU, K % 16 == 0.
    NaN / Inf input sets BD_DEVERR_NONFINITE in the device error word."""
    if w.dim() != 2:
        raise ValueError("w must be 2-D (N, K)")
    if w.dtype not in _IN:
        raise TypeError(f"w must be float32 or bfloat16, got {w.dtype}")
    _need(w, w.dtype, "w")
    N, K = w.shape
    if K % 16:
        raise ValueError(f"K must be a multiple of 16, got {K}")
    codes = torch.empty((N, K // 2), dtype=torch.uint8, device=w.device)
    scales = torch.empty((N, K // 16), dtype=torch.uint8, device=w.device)
    tstat = torch.empty(2, dtype=torch.int32, device=w.device)
    call("bd_quantize_b_nvfp4", _p(w), _IN[w.dtype], _p(codes), _p(scales), _p(tstat), N, K,
         _stream(stream))
    return codes, scales, tstat


def tensor_scale_of(tstat: torch.Tensor) -> float:
    """The fp32 tensor scale held in tstat[0] (reads it back to the host)."""
    return float(tstat[:1].view(torch.float32).item())


def quantize_weights(w: torch.Tensor, stream=None) -> PackedWeights:
    """Weights w (N, K) fp32/bf16 -> PackedWeights (NVFP4 quantised on the GPU, then tiled for
    the GEMM). N % 128 == 0, K % 128 == 0. Reads the tensor scale back to the host once."""
    codes, scales, tstat = quantize_nvfp4(w, stream)
    return pack_weights(codes, scales, tensor_scale_of(tstat), stream)


def query_workspace(M: int, N: int, K: int, split_k: int = 0, split_mode: str = "reduce") -> int:
    return int(_lib.load().bd_query_workspace(M, N, K, split_k, SPLIT_MODES[split_mode]))


# Incremented whenever device_error() finds a bounded wait that ran out: a GEMM that gave up
# mid-call can leave stream-K arrival counters set, so every Workspace re-zeroes before its
# next use.
_ws_epoch = 0


def _note_device_error(word: int) -> None:
    global _ws_epoch
    if word & _lib.BD_DEVERR_WAIT_MASK:
        _ws_epoch += 1


class Workspace:
    """Device scratch for bd_w4a6_gemm. Zeroed when allocated, whenever the problem shape
    changes, and after device_error() reported a bounded wait that ran out (an aborted call
    can leave its stream-K counters set); between calls of one shape the counters are left at
    zero by the kernel itself, so repeated calls (and CUDA-graph replays) need no clearing.
    The zeroing is ordered on the stream the GEMM runs on. One per stream."""

    def __init__(self, device=None):
        self.buf = None
        self.device = device
        self.key = None
        self.epoch = _ws_epoch

    def get(self, nbytes: int, device, key=None, stream=None) -> Optional[torch.Tensor]:
        if nbytes == 0:
            return None
        device = torch.device(device)
        if device.type == "cuda" and stream is not None and not hasattr(stream, "cuda_stream"):
            stream = torch.cuda.ExternalStream(int(stream), device=device)
        ctx = torch.cuda.stream(stream) if (device.type == "cuda" and stream is not None) \
            else _nullctx()
        with ctx:
            if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
                self.buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            elif key != self.key or self.epoch != _ws_epoch:
                self.buf[:nbytes].zero_()
        self.key = key
        self.epoch = _ws_epoch
        return self.buf


class _nullctx:
    def __enter__(self):
        return None

    def __exit__(self, *a):
        return False


_default_ws = {}


def _workspace_for(device, stream) -> Workspace:
    key = (str(device), int(_stream(stream).value or 0))
    if key not in _default_ws:
        _default_ws[key] = Workspace()
    return _default_ws[key]


def w4a6_gemm(acts: PackedActivations, weights: PackedWeights,
              bias: Optional[torch.Tensor] = None, out_dtype=torch.bfloat16,
              epilogue: str = "none", split_k: int = 0, split_mode: str = "reduce",
              out: Optional[torch.Tensor] = None, workspace=None,
              stream=None, overlap_prev: bool = False,
              weights_static: bool = False, single_cta: bool = False) -> torch.Tensor:
    """C[M, N] = A . B^T * tensor_scale (+ bias, activation) on the tensor cores.

    split_k=0 (default) runs the persistent stream-K schedule; its scratch comes from
    `workspace` (a zeroed uint8 tensor or a Workspace), else from a per-stream Workspace.
    overlap_prev: the kernel may be scheduled while the previous kernel on the stream
    finishes (it waits for it before reading A/bias or writing C). weights_static (with
    overlap_prev): the previous kernel does not write the weights, so they stream early.
    single_cta: no CTA-pair tiles (large GEMMs otherwise compute 256-token tiles on pairs of
    CTAs sharing each MMA; same results)."""
    M, K, N = acts.M, acts.K, weights.N
    if weights.K != K:
        raise ValueError(f"K mismatch: activations {K}, weights {weights.K}")
    planes = split_k if (split_mode == "planes" and split_k > 1) else 1
    if out is None:
        shape = (planes, M, N) if planes > 1 else (M, N)
        alloc = torch.zeros if split_mode == "atomic" else torch.empty
        out = alloc(shape, dtype=out_dtype, device=acts.codes.device)
    _need(out, out_dtype, "out", planes * M * N)
    ws_bytes = query_workspace(M, N, K, split_k, split_mode)
    key = (M, N, K, split_k, split_mode)
    if isinstance(workspace, Workspace):
        workspace = workspace.get(ws_bytes, acts.codes.device, key, stream)
    elif workspace is None and ws_bytes:
        workspace = _workspace_for(acts.codes.device, stream).get(ws_bytes, acts.codes.device,
                                                                  key, stream)
    if bias is not None:
        _need(bias, torch.bfloat16, "bias", N)
    epi = EPILOGUES[epilogue]
    if epi != _lib.BD_EPI_NONE and bias is None:
        raise ValueError(f"epilogue {epilogue!r} needs a bias")
    flags = (_lib.BD_GEMM_OVERLAP_PREV if overlap_prev else 0) | \
        (_lib.BD_GEMM_WEIGHTS_STATIC if weights_static else 0) | \
        (_lib.BD_GEMM_B_E4M3 if weights.sideband == "e4m3" else 0) | \
        (_lib.BD_GEMM_SINGLE_CTA if single_cta else 0)
    call("bd_w4a6_gemm_ex", _p(out), _p(acts.codes), _p(acts.scales), _p(weights.codes),
         _p(weights.scales), float(weights.tensor_scale), _p(bias), M, N, K, split_k,
         SPLIT_MODES[split_mode], _OUT[out_dtype], epi, _p(workspace),
         0 if workspace is None else workspace.numel() * workspace.element_size(),
         flags, _stream(stream))
    return out


def w4a6_linear(x: torch.Tensor, weights: PackedWeights, bias: Optional[torch.Tensor] = None,
                out_dtype=torch.bfloat16, epilogue: str = "none", out: Optional[torch.Tensor] = None,
                workspace=None, stream=None) -> torch.Tensor:
    """C = quantise_mxfp6(x) . W^T * tensor_scale (+ bias, activation) from raw activations x
    (M, K) fp32/bf16 on the GPU: the on-device MXFP6 quantiser, then the W4A6 GEMM, both
    launched with programmatic serialisation: the quantiser starts as the previous kernel on the
    stream ends, and the GEMM's CTAs take the SMs the quantiser leaves free and stream the
    (static) weights while it finishes; each reads its inputs only after its predecessor."""
    acts = quantize_activations(x, stream, overlap_prev=True)
    return w4a6_gemm(acts, weights, bias=bias, out_dtype=out_dtype, epilogue=epilogue, out=out,
                     workspace=workspace, stream=stream, overlap_prev=True, weights_static=True)


def w4a6_gemm_noalloc(acts: PackedActivations, weights: PackedWeights, out: torch.Tensor,
                      bias: Optional[torch.Tensor] = None, epilogue: str = "none",
                      stream=None) -> torch.Tensor:
    """w4a6_gemm (default schedule) through bd_w4a6_gemm_noalloc: no workspace and no device
    allocation on this path (`out` is the caller's); its scratch is a static array in the
    library shared by every call on the device, so calls must not overlap in time."""
    M, K, N = acts.M, acts.K, weights.N
    if weights.K != K:
        raise ValueError(f"K mismatch: activations {K}, weights {weights.K}")
    if out.dtype not in _OUT:
        raise ValueError(f"unsupported output dtype {out.dtype}")
    if weights.sideband != "class":
        raise ValueError("bd_w4a6_gemm_noalloc takes weights packed by bd_pack_b (sideband 'class')")
    _need(out, out.dtype, "out", M * N)
    if bias is not None:
        _need(bias, torch.bfloat16, "bias", N)
    epi = EPILOGUES[epilogue]
    if epi != _lib.BD_EPI_NONE and bias is None:
        raise ValueError(f"epilogue {epilogue!r} needs a bias")
    call("bd_w4a6_gemm_noalloc", _p(out), _p(acts.codes), _p(acts.scales), _p(weights.codes),
         _p(weights.scales), float(weights.tensor_scale), _p(bias), M, N, K, _OUT[out.dtype],
         epi, _stream(stream))
    return out


def mma_peak_tflops(n_cols: int = 256, a_from_tmem: bool = False, mmas_per_cta: int = 1 << 16,
                    reps: int = 3, stream=None, pair: bool = False) -> float:
    """Measured rate of the block-scaled tensor-core MMA the GEMM uses (bd_probe_mma_peak):
    one CTA per SM issuing mmas_per_cta back-to-back tcgen05.mma.kind::mxf8f6f4 of
    M = 128, N = n_cols, K = 32 (pair=True: the CTA-pair MMA, M = 256 over two CTAs, N = 256,
    A from tensor memory), timed with CUDA events on the launching stream after one warm-up
    launch; the best of `reps` launches, in TFLOP/s. The FP6 (= FP8-rate) denominator of the
    GEMM's tensor roofline."""
    if stream is None:
        stream = torch.cuda.current_stream()
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    if pair:
        n_cols, sms = 256, sms // 2 * 2
    args = (int(mmas_per_cta), int(n_cols), 2 if pair else (1 if a_from_tmem else 0),
            _stream(stream))
    call("bd_probe_mma_peak", *args)
    best = None
    for _ in range(max(1, reps)):
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        call("bd_probe_mma_peak", *args)
        t1.record(stream)
        t1.synchronize()
        ms = t0.elapsed_time(t1)
        best = ms if best is None else min(best, ms)
    if device_error(clear=True) != 0:
        raise RuntimeError("the MMA peak probe reported a device error")
    flops = sms * float(mmas_per_cta) * 2.0 * 128 * n_cols * 32
    return flops / (best / 1e3) / 1e12


def device_error(clear: bool = True) -> int:
    """Error word set by the library's kernels (0 = none): bits 0..4 a bounded wait of the
    GEMM ran out, BD_DEVERR_NONFINITE (0x20) the quantiser saw NaN / Inf."""
    w = ctypes.c_uint32(0)
    call("bd_device_error", ctypes.byref(w), 1 if clear else 0)
    _note_device_error(int(w.value))
    return int(w.value)


def selftest_bounded_wait(limit_cycles: int = 2_000_000, stream=None) -> int:
    """Run the bounded-wait diagnostic kernel (bd_selftest_bounded_wait) and return the device
    error word it leaves, clearing it: BD_DEVERR_WAIT_TMA when the waits behave."""
    if device_error(clear=True) != 0:
        raise RuntimeError("device error word already set before the self-test")
    call("bd_selftest_bounded_wait", int(limit_cycles), _stream(stream))
    return device_error(clear=True)
