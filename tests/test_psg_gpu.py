"""The drop-in operator `compile_preshuffle_gemm_a8` driven the way the reference's own scripts
drive it: kernel/verify_w4a6.py (constant operands, C = K*a*b*b_scale, async/no-async and
split cross-checks) and kernel/bench_sweep.py (random bytes, the reference's buffer sizes,
the no-output guard, split_k planes summed by the caller, atomic split into a zeroed fp32 C)."""
import numpy as np
import pytest

import w4a6_oracle as o

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


class VoidPtr:
    """Stand-in for flydsl's from_c_void_p(dtype, ptr) argument objects (.value)."""

    def __init__(self, t):
        self.value = t.data_ptr()


def ref_buffers(M, N, K, dev="cuda"):
    """Buffers sized exactly as kernel/verify_w4a6.py:100-106 and bench_sweep.py:59-85."""
    sa = torch.zeros((M * K) // 32 * 2 + 4096, dtype=torch.uint8, device=dev)
    sb = torch.zeros((N * K) // 32 * 2 + 4096, dtype=torch.uint8, device=dev)
    bias = torch.zeros((N,), dtype=torch.bfloat16, device=dev)
    lut = torch.zeros(8 * 256, dtype=torch.int32, device=dev)
    return sa, sb, bias, lut


@pytest.mark.parametrize("a_val,a_byte", [(3.25, 0x55), (-1.25, 0xAA), (-7.5, 0xFF), (0.0, 0x00)])
@pytest.mark.parametrize("b_val", [2.0, 0.5, 6.0])
@pytest.mark.parametrize("b_scale,b_byte", [(1.0, 0x38), (2.0, 0x40), (1.5, 0x3C)])
def test_verify_w4a6_byte_uniform(a_val, a_byte, b_val, b_scale, b_byte):
    """verify_w4a6.py --dtype w6a6_tc --a_uniform_byte: expected = K*a_val*b_val*b_scale,
    pass at |err| <= 1e-3*|expected| (:185-192). The buffers are filled the way the script
    fills them -- constant code and scale bytes straight into the reference-sized buffers, no
    packer -- which the operator reads as the reference does."""
    from bitdance_b200.psg import compile_preshuffle_gemm_a8
    M, N, K = 128, 256, 2048
    sa, sb, bias, lut = ref_buffers(M, N, K)
    a = torch.full((M, K), a_byte, dtype=torch.uint8, device="cuda")
    bc = o.E2M1_POS.tolist().index(b_val)
    b_nat = torch.full((N, K // 2), (bc << 4) | bc, dtype=torch.uint8, device="cuda")
    sa.fill_(127)
    b = b_nat
    sb.fill_(b_byte)
    c = torch.zeros((M, N), dtype=torch.bfloat16, device="cuda")
    launch = compile_preshuffle_gemm_a8(M=M, N=N, K=K, tile_m=128, tile_n=256, tile_k=128,
                                        in_dtype="w6a6_tc", out_dtype="bf16")
    launch(VoidPtr(c), VoidPtr(a), VoidPtr(b), VoidPtr(sa), VoidPtr(sb), VoidPtr(bias),
           VoidPtr(lut), M, N, torch.cuda.current_stream())
    torch.cuda.synchronize()
    C = c.float().cpu().numpy()
    # the transcode folds the scale mantissa into the codes; for these operands it is exact
    expected = K * a_val * b_val * b_scale
    assert np.abs(C - expected).max() <= 1e-3 * abs(expected) + (1e-6 if expected == 0 else 0)


def _random_launch(M, N, K, split_k, split_reduce, seed=0):
    from bitdance_b200.psg import compile_preshuffle_gemm_a8
    import bitdance_b200 as bd
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    sa, sb, bias, lut = ref_buffers(M, N, K)
    a_nat = torch.randint(0, 64, (M, K), dtype=torch.uint8, device="cuda", generator=g)
    e8_nat = torch.randint(122, 132, (M, K // 32), dtype=torch.uint8, device="cuda", generator=g)
    b_nat = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
    s_nat = torch.randint(0x30, 0x48, (N, K // 16), dtype=torch.uint8, device="cuda", generator=g)
    acts = bd.pack_activations(a_nat, e8_nat)
    w = bd.pack_weights(b_nat, s_nat, sideband="e4m3")
    sa[: acts.scales.numel()].copy_(acts.scales)
    sb[: w.scales.numel()].copy_(w.scales)
    if split_reduce == "atomic":
        c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    else:
        c = torch.zeros((split_k, M, N), dtype=torch.bfloat16, device="cuda")
    launch = compile_preshuffle_gemm_a8(M=M, N=N, K=K, tile_m=128, tile_n=256, tile_k=128,
                                        in_dtype="w4a6_tc", out_dtype="bf16", split_k=split_k,
                                        split_reduce=split_reduce)
    launch(c, acts.codes, w.codes, sa, sb, bias, lut, M, N, torch.cuda.current_stream(),
           b_tensor_scale=0.25)
    torch.cuda.synchronize()
    e6, e8 = o.transcode_b(b_nat.cpu().numpy(), s_nat.cpu().numpy(), 16)
    gold = o.gemm_gold(a_nat.cpu().numpy(), e8_nat.cpu().numpy(), e6, e8, 0.25)
    out = c.float().sum(0) if split_reduce != "atomic" else c
    return out.cpu().numpy(), gold


@pytest.mark.parametrize("split_k,split_reduce", [(1, "planes"), (4, "planes"), (8, "planes"),
                                                  (1, "atomic"), (4, "atomic")])
def test_bench_sweep_flow(split_k, split_reduce):
    """bench_sweep.py: random operands, the output must not be all zero (:297-326), the caller
    sums the split planes (:141-142) or zeroes an fp32 C for atomics (:134-140)."""
    got, gold = _random_launch(128, 512, 2048, split_k, split_reduce)
    assert np.abs(got).max() > 0
    assert o.rel_linf(gold, got) <= 1e-2


def test_split_k_matches_unsplit():
    """verify_w4a6-style cross-check: the split result equals the unsplit one (to fp32 order)."""
    a, gold = _random_launch(64, 256, 4096, 1, "atomic", seed=3)
    b, _ = _random_launch(64, 256, 4096, 8, "atomic", seed=3)
    assert np.abs(a - b).max() <= 1e-5 * np.abs(gold).max()


def _e4m3_of_e8m0(e):
    s = int(e) - 127
    if -6 <= s <= 8:
        return (s + 7) << 3
    if -9 <= s <= -7:
        return 0x04 >> (-7 - s)
    return 0


def test_e8m0_to_e4m3_pairs_every_byte():
    """bd_scales_e8m0_to_e4m3_pairs over all 256 E8M0 bytes: the E4M3 byte of the same power of
    two, duplicated for both 16-blocks; bytes without an E4M3 form give 0 and BD_DEVERR_RANGE."""
    import bitdance_b200 as bd
    from bitdance_b200 import _lib
    from bitdance_b200._lib import call
    assert bd.device_error() == 0
    e8 = torch.arange(256, dtype=torch.uint8, device="cuda")
    out = torch.full((512,), 0xEE, dtype=torch.uint8, device="cuda")
    call("bd_scales_e8m0_to_e4m3_pairs", e8.data_ptr(), out.data_ptr(), 256, None)
    got = out.cpu().numpy().reshape(256, 2)
    want = np.array([_e4m3_of_e8m0(e) for e in range(256)], np.uint8)
    assert np.array_equal(got[:, 0], want) and np.array_equal(got[:, 1], want)
    assert bd.device_error() == _lib.BD_DEVERR_RANGE
    # in range only: no error
    call("bd_scales_e8m0_to_e4m3_pairs", e8[118:136].data_ptr(), out.data_ptr(), 18, None)
    assert bd.device_error() == 0


@pytest.mark.parametrize("split_k,split_reduce", [(1, "planes"), (4, "planes"), (4, "atomic")])
def test_w4a6_arm_is_bit_exact_with_the_transcode_arm(split_k, split_reduce):
    """kernel/verify_w4a6.py:166-172: with power-of-two weight scales, the MXFP4 arm ("w4a6",
    E8M0 per-32 scales) and the NVFP4 transcode arm ("w6a6_tc", the same powers of two as E4M3
    bytes) give bit-identical C (fp32 atomics add partials in no fixed order, so that mode is
    compared within the tolerance); both match the MXFP4 gold (E2M1 x 2^(e-127))."""
    from bitdance_b200.psg import compile_preshuffle_gemm_a8
    import bitdance_b200 as bd
    M, N, K = 64, 512, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    a_nat = torch.randint(0, 64, (M, K), dtype=torch.uint8, device="cuda", generator=g)
    a_e8 = torch.randint(122, 132, (M, K // 32), dtype=torch.uint8, device="cuda", generator=g)
    b_nat = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
    e8 = torch.randint(118, 136, (N, K // 32), dtype=torch.uint8, device="cuda", generator=g)
    acts = bd.pack_activations(a_nat, a_e8)
    # the NVFP4 form of the same weights: both 16-blocks carry the power of two as E4M3
    lut = torch.tensor([_e4m3_of_e8m0(e) for e in range(256)], dtype=torch.uint8, device="cuda")
    s16 = lut[e8.long()].repeat_interleave(2, dim=1).contiguous()
    w = bd.pack_weights(b_nat, s16, sideband="e4m3")
    # the MXFP4 arm's scale buffer: one E8M0 byte per 32-block, in the sideband's block order
    # (the E8M0 bytes regrouped by the same packer, taking the first byte of each pair)
    w8 = bd.pack_weights(b_nat, e8.repeat_interleave(2, dim=1).contiguous(), sideband="e4m3")
    tiled_e8 = w8.scales.view(-1, 2)[:, 0].contiguous()
    outs = {}
    for dtype, sb in (("w6a6_tc", w.scales), ("w4a6", tiled_e8)):
        launch = compile_preshuffle_gemm_a8(M=M, N=N, K=K, tile_m=128, tile_n=256, tile_k=128,
                                            in_dtype=dtype, out_dtype="bf16", split_k=split_k,
                                            split_reduce=split_reduce)
        if split_reduce == "atomic":
            c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        else:
            c = torch.zeros((split_k, M, N), dtype=torch.bfloat16, device="cuda")
        launch(c, acts.codes, w.codes, acts.scales, sb, None, None, M, N, None)
        torch.cuda.synchronize()
        outs[dtype] = c
    assert bd.device_error() == 0
    if split_reduce == "atomic":
        diff = (outs["w6a6_tc"] - outs["w4a6"]).abs().max().item()
        assert diff <= 1e-5 * outs["w6a6_tc"].abs().max().item()
    else:
        assert torch.equal(outs["w6a6_tc"], outs["w4a6"])
    # gold: MXFP4 weights dequantised directly
    codes = o.unpack_nibbles(b_nat.cpu().numpy()).astype(np.int64)
    wv = np.where(codes & 8, -1.0, 1.0) * o.E2M1_POS[codes & 7]
    wv *= np.repeat(np.exp2(e8.cpu().numpy().astype(np.float64) - 127), 32, axis=1)
    av = o.dequant_operand(a_nat.cpu().numpy(), a_e8.cpu().numpy())
    gold = av @ wv.T
    got = outs["w4a6"].float()
    got = (got.sum(0) if got.dim() == 3 else got).cpu().numpy()
    assert o.rel_linf(gold, got) <= 1e-2
