"""Helpers for GEMM parity at the BASELINE configs' full sizes (test infrastructure).

The operands are drawn on the GPU from a seeded torch generator with each config's
distribution (normal, Student-t, outlier-channel activations), quantised by the library's
device quantisers, and checked in three steps:

* the quantised bytes of sampled weight and token rows equal the CPU oracle's quantisation of
  the same fp32 values, bit for bit (the oracle is pinned to the reference's own outputs);
* the GEMM output of sampled token rows (at least one per token tile, all N columns) is
  compared with an fp64 accumulation of the dequantised operands, where the weights are
  transcoded and dequantised by the C restatement of the reference codec (oracle/liborc.so),
  at max-abs-rel error <= 1e-2 and an elementwise bound at bf16 resolution;
* for the full-size check to stay a few seconds of CPU per case, only the sampled token rows
  go through the gold.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

import w4a6_oracle as o

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL_REL_LINF = 1e-2


def _orc():
    import subprocess
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
    return lib


_LIB = None


def orc():
    global _LIB
    if _LIB is None:
        _LIB = _orc()
    return _LIB


def threads():
    return max(1, min(16, os.cpu_count() or 1))


# ----------------------------------------------------------------------------------------
# seeded synthetic operands on the GPU

def gen(torch, kind: str, shape, seed: int, std: float = 1.0):
    """fp32 tensor on cuda:0. kind: "normal" (N(0, std)), "t" (Student-t df=5 scaled to std),
    "outlier" (N(0,1) with 0.1% of the K channels times 20)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    if kind == "normal":
        return torch.randn(shape, device="cuda", generator=g) * std
    if kind == "t":
        z = torch.randn(shape, device="cuda", generator=g)
        chi = torch.zeros(shape, device="cuda")
        for _ in range(5):
            chi += torch.randn(shape, device="cuda", generator=g).square()
        return z / torch.sqrt(chi / 5.0) * (std / float(np.sqrt(5.0 / 3.0)))
    if kind == "outlier":
        x = torch.randn(shape, device="cuda", generator=g)
        ch = torch.rand(shape[-1], device="cuda", generator=g) < 0.001
        return torch.where(ch[None, :], x * 20.0, x)
    raise ValueError(kind)


class Weights:
    """N x K weights drawn on the GPU, NVFP4-quantised by the device quantiser and packed for
    the GEMM; the natural-layout bytes are kept on the host for the gold."""

    def __init__(self, torch, N, K, kind, std, seed):
        import bitdance_b200 as bd
        self.N, self.K = N, K
        w = gen(torch, kind, (N, K), seed, std)
        self.packed, self.sc, tstat = bd.quantize_nvfp4(w)
        self.s_t = bd.tensor_scale_of(tstat)
        self.amax = float(w.abs().max().item())
        self.rows = sample_rows(N, 64, seed)
        self.sample = w[torch.as_tensor(self.rows, device="cuda")].cpu().numpy()
        del w
        self.gemm = bd.pack_weights(self.packed, self.sc, self.s_t)
        self.host_packed = self.packed.cpu().numpy()
        self.host_sc = self.sc.cpu().numpy()

    def check(self):
        """The device quantiser's bytes of the sampled rows equal the oracle's, and the tensor
        scale is the oracle's formula applied to the tensor's amax."""
        s_t = o.tensor_scale(np.array([self.amax], np.float32))
        assert np.float32(self.s_t) == s_t
        sb, c = o.encode_nvfp4((self.sample / s_t).reshape(-1), block=16)
        r = self.rows
        assert np.array_equal(self.host_sc[r], sb.reshape(len(r), -1))
        assert np.array_equal(self.host_packed[r], o.pack_nibbles(c.reshape(len(r), -1)))


class Acts:
    """M x K activations drawn on the GPU, MXFP6-quantised by the device quantiser."""

    def __init__(self, torch, M, K, kind, seed):
        import bitdance_b200 as bd
        self.M, self.K = M, K
        x = gen(torch, kind, (M, K), seed)
        self.codes, self.e8 = bd.quantize_mxfp6(x)
        self.rows = token_rows(M)
        idx = torch.as_tensor(self.rows, device="cuda")
        self.sample = x[idx].cpu().numpy()
        del x
        self.gemm = bd.pack_activations(self.codes, self.e8)
        self.host_codes = self.codes[idx].cpu().numpy()
        self.host_e8 = self.e8[idx].cpu().numpy()

    def check(self):
        codes, e8 = o.quantize_a_mxfp6(self.sample)
        assert np.array_equal(self.host_codes, codes)
        assert np.array_equal(self.host_e8, e8)


def gold_rows(acts: Acts, w: Weights, bias=None):
    """(C, Cabs) of the sampled token rows: fp64 accumulation of the dequantised operands,
    the weights transcoded by the C restatement of the reference codec."""
    return gold_from_bytes(acts.host_codes, acts.host_e8, w.host_packed, w.host_sc, w.s_t, bias)


def gemm_rows(torch, out, acts: Acts):
    return out[torch.as_tensor(acts.rows, device="cuda")].float().cpu().numpy()


def sample_rows(n, k, seed):
    if n <= k:
        return np.arange(n)
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(n, k, replace=False))


def token_rows(M, per_tile=2, tile=128):
    """All rows for a decode batch; otherwise the first and last row of every 128-row token
    tile (every tile of the GEMM's schedule is looked at)."""
    if M <= 64:
        return np.arange(M)
    rows = set()
    for t0 in range(0, M, tile):
        rows.add(t0)
        rows.add(min(M, t0 + tile) - 1)
        if per_tile > 2:
            rows.add(t0 + (tile // 2 if t0 + tile // 2 < M else 0))
    return np.array(sorted(rows))


def gold_from_bytes(a_codes, a_e8, b_packed, b_sc, s_t, bias=None, chunk=4096):
    """C = deq(A) . deq(transcode(B))^T * s_t (+ bias) in fp64 for the given token rows, and
    the same with magnitudes only (for the elementwise bound)."""
    lib = orc()
    N, Kh = b_packed.shape
    K = 2 * Kh
    A = o.dequant_operand(np.asarray(a_codes, np.uint8), np.asarray(a_e8, np.uint8))
    Aabs = np.abs(A)
    b_packed = np.ascontiguousarray(b_packed, np.uint8)
    b_sc = np.ascontiguousarray(b_sc, np.uint8)
    C = np.empty((A.shape[0], N))
    Cabs = np.empty((A.shape[0], N))
    ch = min(chunk, N)
    e6 = np.empty(ch * K, np.uint8)
    e8 = np.empty(ch * K // 32, np.uint8)
    Bf = np.empty((ch, K), np.float32)
    for r0 in range(0, N, ch):
        r1 = min(N, r0 + ch)
        nb = (r1 - r0) * K // 32
        assert lib.orc_transcode(b_packed[r0:r1].ctypes.data, b_sc[r0:r1].ctypes.data, nb, 16,
                                 e6.ctypes.data, e8.ctypes.data, threads()) == 0
        assert lib.orc_dequant(e6.ctypes.data, e8.ctypes.data, nb, Bf.ctypes.data,
                               threads()) == 0
        B = Bf[: r1 - r0].astype(np.float64)
        C[:, r0:r1] = A @ B.T
        Cabs[:, r0:r1] = Aabs @ np.abs(B).T
    C *= float(s_t)
    Cabs *= abs(float(s_t))
    if bias is not None:
        C += np.asarray(bias, np.float64)[None, :]
    return C, Cabs


def check_rows(got_rows, C, Cabs, ulp=2.0 ** -8):
    """max-abs-rel <= 1e-2 and |got - C| <= ulp |C| + 2^-20 Cabs
    elementwise (bf16 rounding of C plus fp32 accumulation-order differences)."""
    g = np.asarray(got_rows, np.float64)
    assert np.isfinite(g).all()
    assert np.abs(g).max() > 0, "kernel wrote no output"
    assert o.rel_linf(C, g) <= TOL_REL_LINF
    bound = ulp * np.abs(C) + 2.0 ** -20 * Cabs + 1e-30
    bad = np.abs(g - C) > bound
    assert not bad.any(), f"{bad.sum()} elements outside bound; first at {np.argwhere(bad)[0]}"
