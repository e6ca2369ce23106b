"""The on-device NVFP4 weight quantiser (bd_quantize_b_nvfp4) against the oracle's
quantize_b_nvfp4, the reference's two-level NVFP4 encode (remote/quant_real_weights.py:273-287,
kernel/nvfp4_codec.py:34-63).

CPU: the kernel's float32 formulation (block scale = __fdiv_ru(amax, 6) rounded up to a 3-bit
mantissa, codes by exact comparisons against midpoint * scale) restated in numpy equals the
fp64 oracle on adversarial tensors (exact ties, block maxima at exactly 6 * scale and one ulp
either side, zero blocks, both scale clamps); the C ABI rejects bad arguments. GPU: the kernel
is bit-exact against the oracle for fp32 and bf16 input, quantize_weights feeds the GEMM, and
NaN / Inf set the device error bit."""
import ctypes

import numpy as np
import pytest

import w4a6_oracle as o

E2M1_MID = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)


def adversarial_weights(seed: int = 0, rows: int = 64, K: int = 256) -> np.ndarray:
    """(rows, K) float32 weights stressing each step of the rule. Even seeds: the tensor
    maximum is 2688 * 2^-10, so s_t = 2^-10 exactly and the grid points and midpoints of rows
    0..7 stay exact ties after the tensor scale. Odd seeds: a maximum whose s_t rounds so that
    the top block's amax exceeds 6 * 448 (block scale clamped at 448)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_t(5, (rows, K)) * 0.02).astype(np.float32)
    blk = w.reshape(rows, K // 16, 16)
    # rows 0..7: blocks of exact E2M1 grid points and midpoints times an E4M3 scale
    grid = np.array([0, .25, .5, .75, 1, 1.25, 1.5, 1.75, 2, 2.5, 3, 3.5, 4, 5, 6, 6], np.float32)
    for r in range(8):
        for b in range(K // 16):
            sc = np.float32((1 + (b % 8) / 8) * 2.0 ** (b % 9 - 12))
            sgn = np.where(rng.random(16) < 0.5, -1, 1).astype(np.float32)
            blk[r, b] = grid * sc * sgn
    # rows 8..9: block maxima at 6 * scale exactly, and one float32 ulp either side
    for r in (8, 9):
        for b in range(K // 16):
            m = np.float32(6 * (1 + (b % 8) / 8) * 2.0 ** (b % 7 - 10))
            m = [m, np.nextafter(m, np.float32(0)), np.nextafter(m, np.float32(1))][b % 3]
            blk[r, b] = rng.uniform(-1, 1, 16).astype(np.float32) * m / 2
            blk[r, b, b % 16] = m if r == 8 else -m
    # row 10: zero blocks and signed zeros; row 11: tiny values (scale clamps at 2^-6)
    blk[10] = 0.0
    blk[10, 1, ::2] = -0.0
    blk[11] = (rng.standard_normal((K // 16, 16)) * 1e-9).astype(np.float32)
    # row 12: the tensor maximum (one element) and its float32 predecessor
    top = np.float32(2688.0 * 2.0 ** -10) if seed % 2 == 0 else np.float32(7.123)
    blk[12, 0, 0] = top
    blk[12, 1, 0] = np.nextafter(top, np.float32(0))
    return blk.reshape(rows, K)


def kernel_rule(w: np.ndarray):
    """The kernel's steps (quantize_b.cuh), restated in numpy for a CPU check of the exactness
    argument. Test-side only. Returns (codes (N, K) nibbles, scale bytes (N, K/16), s_t)."""
    w = np.asarray(w, np.float32)
    N, K = w.shape
    amax = np.float32(np.max(np.abs(w)))
    s_t = np.float32(1.0) if amax == 0 else np.float32(np.float64(amax) / 2688.0)
    v = (w / s_t).astype(np.float32).reshape(-1, 16)
    bam = np.max(np.abs(v), axis=1)
    # smallest float32 >= bam / 6 (exact comparisons in float64)
    q = (bam.astype(np.float64) / 6.0).astype(np.float32)
    up = q.astype(np.float64) * 6.0 < bam.astype(np.float64)
    q = np.where(up, np.nextafter(q, np.float32(np.inf)), q)
    b = q.view(np.uint32).astype(np.int64)
    b = np.where(b & 0xFFFFF, (b | 0xFFFFF) + 1, b)
    b = np.clip(b, 0x3C800000, 0x43E00000)
    B = b.astype(np.uint32).view(np.float32)
    byte = ((((b >> 23) - 127 + 7) << 3) | ((b >> 20) & 7)).astype(np.uint8)
    zero = bam == 0
    B = np.where(zero, np.float32(1.0), B)
    byte = np.where(zero, np.uint8(0x38), byte)
    t = (E2M1_MID[None, :] * B[:, None]).astype(np.float32)          # exact products
    idx = (np.abs(v)[:, :, None] > t[:, None, :]).sum(axis=2)
    sign = (v < 0) & (idx != 0)
    codes = (idx | (sign.astype(np.int64) << 3)).astype(np.uint8)
    return codes.reshape(N, K), byte.reshape(N, K // 16), s_t


def test_kernel_rule_equals_oracle():
    for seed in range(3):
        w = adversarial_weights(seed)
        gc, gs, gt = o.quantize_b_nvfp4(w, block=16)
        kc, ks, kt = kernel_rule(w)
        assert kt == gt
        assert np.array_equal(ks, gs)
        assert np.array_equal(kc, gc)


def test_kernel_rule_equals_oracle_on_bf16_values_and_zero_tensor():
    torch = pytest.importorskip("torch")
    w = torch.from_numpy(adversarial_weights(4)).to(torch.bfloat16).float().numpy()
    gc, gs, gt = o.quantize_b_nvfp4(w, block=16)
    kc, ks, kt = kernel_rule(w)
    assert kt == gt and np.array_equal(ks, gs) and np.array_equal(kc, gc)
    z = np.zeros((4, 32), np.float32)
    assert [np.array_equal(a, b) for a, b in zip(kernel_rule(z)[:2], o.quantize_b_nvfp4(z)[:2])] \
        == [True, True]


def test_quantize_b_rejects_bad_arguments():
    from bitdance_b200 import build
    build.build_library()
    from bitdance_b200 import _lib
    lib = _lib.load()
    P = ctypes.c_void_p
    ok = P(4096)  # never dereferenced: validation fails first
    q = lib.bd_quantize_b_nvfp4
    assert q(ok, 3, ok, ok, ok, 4, 128, None) == -1          # unknown dtype
    assert q(ok, 0, ok, ok, None, 4, 128, None) == -1        # no tstat
    assert q(ok, 0, ok, ok, ok, 4, 40, None) == -2           # K % 16
    assert q(ok, 1, ok, ok, ok, 0, 128, None) == -2          # N <= 0
    assert q(P(4104), 0, ok, ok, ok, 4, 128, None) == -3     # w not 16-byte aligned
    assert q(ok, 0, P(4100), ok, ok, 4, 128, None) == -3     # codes not 8-byte aligned


# ---------------------------------------------------------------------------------------
# GPU


def _gpu_vs_oracle(w_np, dtype):
    import torch
    import bitdance_b200 as bd
    w = torch.from_numpy(w_np).to(getattr(torch, dtype)).cuda()
    codes, scales, tstat = bd.quantize_nvfp4(w)
    gc, gs, gt = o.quantize_b_nvfp4(w.float().cpu().numpy(), block=16)
    assert bd.tensor_scale_of(tstat) == float(gt)
    assert np.array_equal(scales.cpu().numpy(), gs)
    assert np.array_equal(codes.cpu().numpy(), o.pack_nibbles(gc))
    assert bd.device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("seed", [0, 1])
def test_gpu_bit_exact_adversarial(dtype, seed):
    _gpu_vs_oracle(adversarial_weights(seed), dtype)


@pytest.mark.gpu
@pytest.mark.parametrize("N,K", [(1, 16), (3, 48), (128, 4096), (300, 1024)])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_gpu_bit_exact_student_t(N, K, dtype):
    _gpu_vs_oracle(o.gen_student_t((N, K), 0.02, N + K), dtype)


@pytest.mark.gpu
def test_gpu_zero_tensor():
    _gpu_vs_oracle(np.zeros((8, 64), np.float32), "float32")


@pytest.mark.gpu
def test_gpu_quantize_weights_feeds_the_gemm():
    """fp32 weights -> GPU NVFP4 -> tiled -> GEMM equals the oracle GEMM on the oracle's own
    quantisation of the same weights."""
    import torch
    import bitdance_b200 as bd
    M, N, K = 16, 512, 1024
    w = o.gen_student_t((N, K), 0.02, 9)
    x = o.gen_normal((M, K), 1.0, 10)
    a_codes, a_e8 = o.quantize_a_mxfp6(x)
    wts = bd.quantize_weights(torch.from_numpy(w).cuda())
    acts = bd.pack_activations(torch.from_numpy(a_codes).cuda(), torch.from_numpy(a_e8).cuda())
    C = bd.w4a6_gemm(acts, wts).float().cpu().numpy()
    b_codes, b_sc, s_t = o.quantize_b_nvfp4(w, block=16)
    assert wts.tensor_scale == float(s_t)
    e6, e8 = o.transcode_b(o.pack_nibbles(b_codes), b_sc, 16)
    assert o.rel_linf(o.gemm_gold(a_codes, a_e8, e6, e8, float(s_t)), C) <= 1e-2


@pytest.mark.gpu
def test_gpu_non_finite_weights_set_the_error_bit():
    import torch
    import bitdance_b200 as bd
    from bitdance_b200 import _lib
    assert bd.device_error() == 0
    for bad in (float("nan"), float("inf")):
        w = torch.randn((4, 64), device="cuda")
        w[1, 17] = bad
        bd.quantize_nvfp4(w)
        assert bd.device_error() == _lib.BD_DEVERR_NONFINITE
