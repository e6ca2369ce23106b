"""The on-device MXFP6 activation quantiser (bd_quantize_a_mxfp6) against the oracle's
quantize_a_mxfp6, the reference's Direct-MXFP6 quantize(x, E8M0, E2M3)
(vector_quant_error.py:283-319 via :389).

CPU: the kernel's formulation (block exponent from the integer amax of the float bits, the
E2M3 index from float bits with a carry-based round-half-down) restated in numpy equals the
fp64 oracle on adversarial blocks (exact
ties, block maxima at exactly 7.5 * 2^e and one ulp either side, the [-40, 40] exponent clamp,
subnormals, signed zeros); the C ABI rejects bad arguments. GPU: the kernel is bit-exact
against the oracle for fp32 and bf16 input, its tiled scales equal bd_pack_a's, a GEMM fed
from it matches the oracle GEMM, and NaN / Inf set the device error bit."""
import ctypes

import numpy as np
import pytest

import w4a6_oracle as o


def adversarial_blocks(seed: int = 0, nrand: int = 512) -> np.ndarray:
    """(nblocks, 32) float32 blocks that stress each step of the rule."""
    rng = np.random.default_rng(seed)
    out = []
    # random blocks over the whole exponent range, including both clamps
    for _ in range(nrand):
        e = rng.integers(-60, 60)
        out.append(rng.standard_normal(32) * np.exp2(float(e)))
    # E2M3 midpoints (exact ties) with the block max pinned at 7.5 * 2^e
    mids = np.concatenate([(np.arange(16) + 0.5) / 8, 2 + (np.arange(8) + 0.5) / 4,
                           4 + (np.arange(7) + 0.5) / 2])
    for e in (-40, -3, 0, 5, 40):
        for sign in (1.0, -1.0):
            blk = np.zeros(32)
            blk[: len(mids)] = sign * mids
            blk[31] = 7.5
            out.append(blk * np.exp2(e))
    # block max at 7.5 * 2^e exactly and one float32 ulp either side
    for e in (-41, -40, -10, 0, 1, 39, 40, 41):
        base = np.float32(7.5 * 2.0 ** e)
        for m in (base, np.nextafter(base, np.float32(0)), np.nextafter(base, np.float32(np.inf))):
            blk = rng.standard_normal(32) * float(m) / 8
            blk[int(rng.integers(32))] = -float(m) if rng.random() < 0.5 else float(m)
            out.append(np.clip(blk, -float(m), float(m)))
    # zero, signed zeros, values that round to code 0 with a negative sign
    out.append(np.zeros(32))
    z = np.zeros(32)
    z[::2] = -0.0
    z[1] = 7.5
    z[3] = -0.06
    z[5] = -0.0625
    out.append(z)
    # subnormal float32 magnitudes, and huge ones (scale clamp at 2^40)
    sub = rng.integers(1, 1 << 23, 32).astype(np.uint32).view(np.float32).astype(np.float64)
    out.append(sub * np.where(rng.random(32) < 0.5, -1, 1))
    out.append(rng.standard_normal(32) * 1e37)
    out.append(np.full(32, -3.0e38))
    while len(out) % 8:  # whole rows of 256 elements
        out.append(np.zeros(32))
    return np.asarray(out, dtype=np.float32)


def kernel_rule(x: np.ndarray):
    """The kernel's steps (quantize_a_kernel in transcode.cuh), restated in numpy for a CPU
    check of the exactness argument: block exponent from the integer amax of |bits|, element
    index ((bits(max(y, z)) + 0x7FFFF) >> 20) - 1008 capped at 31 with y = |x| * 2^-e (float32)
    and z = (y + 1) / 2 rounded up to float32. Test-side only."""
    f = np.asarray(x, dtype=np.float32).reshape(-1, 32)
    ab = f.view(np.uint32) & np.uint32(0x7FFFFFFF)
    amax = ab.max(axis=1).astype(np.int64)
    e = (amax >> 23) - 127 - 2 + ((amax & 0x7FFFFF) > 0x700000)
    e = np.where(amax == 0, 0, np.clip(e, -40, 40))
    inv = np.exp2(-e.astype(np.float64)).astype(np.float32)[:, None]
    y = np.abs(f) * inv                                   # float32 product, exact here
    z64 = (y.astype(np.float64) + 1.0) / 2.0
    z = z64.astype(np.float32)                            # nearest ...
    z = np.where(z.astype(np.float64) < z64, np.nextafter(z, np.float32(np.inf)), z)  # ... up
    t = np.maximum(y, z).view(np.uint32).astype(np.int64)
    mag = np.minimum((t + 0x7FFFF - (1008 << 20)) >> 20, 31)
    sign = (f < 0) & (mag != 0)
    codes = (mag | (sign.astype(np.int64) << 5)).astype(np.uint8)
    return codes.reshape(x.shape), (e + 127).astype(np.uint8).reshape(x.shape[0], -1)


def test_kernel_rule_equals_oracle_on_adversarial_blocks():
    x = adversarial_blocks().reshape(-1, 128)
    gc, ge = o.quantize_a_mxfp6(x)
    kc, ke = kernel_rule(x)
    assert np.array_equal(ke, ge)
    assert np.array_equal(kc, gc)


def test_kernel_rule_equals_oracle_on_bf16_values():
    torch = pytest.importorskip("torch")
    x = torch.from_numpy(adversarial_blocks(1)).to(torch.bfloat16).float().numpy().reshape(-1, 64)
    gc, ge = o.quantize_a_mxfp6(x)
    kc, ke = kernel_rule(x)
    assert np.array_equal(ke, ge) and np.array_equal(kc, gc)


def test_oracle_refuses_non_finite():
    x = np.zeros((1, 32), np.float32)
    x[0, 3] = np.nan
    with pytest.raises(ValueError):
        o.quantize_a_mxfp6(x)


def test_quantize_rejects_bad_arguments():
    from bitdance_b200 import build
    build.build_library()
    from bitdance_b200 import _lib
    lib = _lib.load()
    P = ctypes.c_void_p
    ok = P(4096)  # never dereferenced: validation fails first
    q = lib.bd_quantize_a_mxfp6
    assert q(ok, 2, ok, ok, None, 4, 128, None) == -1        # unknown input dtype
    assert q(None, 0, ok, ok, None, 4, 128, None) == -1      # null x
    assert q(ok, 0, ok, None, None, 4, 128, None) == -1      # no scale output at all
    assert q(ok, 0, ok, ok, None, 4, 48, None) == -2         # K % 32
    assert q(ok, 0, ok, None, ok, 4, 96, None) == -2         # tiled scales need K % 128
    assert q(ok, 1, ok, ok, None, 0, 128, None) == -2        # M <= 0
    assert q(P(4104), 0, ok, ok, None, 4, 128, None) == -3   # x not 16-byte aligned
    assert q(ok, 0, P(4097), ok, None, 4, 128, None) == -3   # codes not 16-byte aligned
    qx = lib.bd_quantize_a_mxfp6_ex
    assert qx(ok, 0, ok, ok, None, 4, 128, 2, None) == -1     # unknown launch flag
    assert qx(ok, 0, ok, ok, None, 4, 48, 1, None) == -2      # then the same checks


# ---------------------------------------------------------------------------------------
# GPU


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_gpu_bit_exact_on_adversarial_blocks(dtype):
    import torch
    import bitdance_b200 as bd
    xs = adversarial_blocks(2).reshape(-1, 256)
    x = torch.from_numpy(xs).to(getattr(torch, dtype)).cuda()
    codes, e8 = bd.quantize_mxfp6(x)
    gc, ge = o.quantize_a_mxfp6(x.float().cpu().numpy())
    assert np.array_equal(e8.cpu().numpy(), ge)
    assert np.array_equal(codes.cpu().numpy(), gc)
    assert bd.device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("M,K", [(1, 32), (3, 96), (5, 128), (16, 4096), (33, 1024),
                                 (257, 2048)])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_gpu_bit_exact_random_shapes(M, K, dtype):
    import torch
    import bitdance_b200 as bd
    g = torch.Generator(device="cuda")
    g.manual_seed(M * 7 + K)
    x = (torch.randn((M, K), generator=g, device="cuda") *
         torch.exp2(torch.randint(-20, 20, (M, 1), generator=g, device="cuda").float()))
    x = x.to(getattr(torch, dtype))
    codes, e8 = bd.quantize_mxfp6(x)
    gc, ge = o.quantize_a_mxfp6(x.float().cpu().numpy())
    assert np.array_equal(e8.cpu().numpy(), ge)
    assert np.array_equal(codes.cpu().numpy(), gc)


@pytest.mark.gpu
@pytest.mark.parametrize("M,K", [(1, 512), (6, 512), (64, 512), (5, 128), (300, 384)])
def test_gpu_tiled_scales_equal_pack_a(M, K):
    """quantize_activations (one launch, tiled scales written directly) == pack_activations of
    the natural outputs, padding rows included."""
    import torch
    import bitdance_b200 as bd
    g = torch.Generator(device="cuda")
    g.manual_seed(M)
    x = torch.randn((M, K), generator=g, device="cuda", dtype=torch.bfloat16)
    packed = bd.quantize_activations(x)
    ref = bd.pack_activations(*bd.quantize_mxfp6(x))
    assert torch.equal(packed.codes, ref.codes)
    assert torch.equal(packed.scales, ref.scales)


@pytest.mark.gpu
def test_gpu_gemm_from_float_activations():
    """x (bf16) -> on-device quantiser -> W4A6 GEMM equals the oracle GEMM of the oracle's
    quantisation of the same x."""
    import torch
    import bitdance_b200 as bd
    M, N, K = 24, 512, 1024
    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b_codes, b_sc, s_t = o.quantize_b_nvfp4(w, block=16)
    b_packed = o.pack_nibbles(b_codes)
    wts = bd.pack_weights(torch.from_numpy(b_packed).cuda(), torch.from_numpy(b_sc).cuda(),
                          float(s_t))
    C = bd.w4a6_gemm(bd.quantize_activations(x.cuda()), wts).float().cpu().numpy()
    a_codes, a_e8 = o.quantize_a_mxfp6(x.float().numpy())
    e6, e8 = o.transcode_b(b_packed, b_sc, 16)
    gold = o.gemm_gold(a_codes, a_e8, e6, e8, float(s_t))
    assert o.rel_linf(gold, C) <= 1e-2


@pytest.mark.gpu
def test_gpu_non_finite_input_sets_the_error_bit():
    """The reference refuses NaN / Inf (vector_quant_error.py:215-252); the kernel flags them in
    the device error word, which the host reads and clears."""
    import torch
    import bitdance_b200 as bd
    from bitdance_b200 import _lib
    assert bd.device_error() == 0
    for bad in (float("nan"), float("inf"), float("-inf")):
        x = torch.randn((4, 128), device="cuda")
        x[2, 77] = bad
        bd.quantize_mxfp6(x)
        assert bd.device_error() == _lib.BD_DEVERR_NONFINITE
    bd.quantize_mxfp6(torch.randn((4, 128), device="cuda"))
    assert bd.device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 16, 200])
def test_gpu_linear_from_raw_activations(M):
    """w4a6_linear (quantiser + programmatically launched GEMM) equals the GEMM of the separately
    quantised activations bit for bit, and the oracle GEMM of the oracle's quantisation."""
    import torch
    import bitdance_b200 as bd
    N, K = 512, 1024
    rng = np.random.default_rng(M)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(torch.bfloat16).cuda()
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    wts = bd.quantize_weights(torch.from_numpy(w).cuda())
    got = bd.w4a6_linear(x, wts)
    ref = bd.w4a6_gemm(bd.quantize_activations(x), wts)
    assert torch.equal(got, ref)
    a_codes, a_e8 = o.quantize_a_mxfp6(x.float().cpu().numpy())
    b_codes, b_sc, s_t = o.quantize_b_nvfp4(w, block=16)
    e6, e8 = o.transcode_b(o.pack_nibbles(b_codes), b_sc, 16)
    gold = o.gemm_gold(a_codes, a_e8, e6, e8, float(s_t))
    assert o.rel_linf(gold, got.float().cpu().numpy()) <= 1e-2
    assert bd.device_error() == 0
