"""The CPU oracle pinned against the reference's own outputs (golden fixtures written by
tests/golden/make_golden.py from scimg/bitdance). CPU only."""
import json
import os

import numpy as np
import pytest

import w4a6_oracle as o
from conftest import GOLDEN, golden, orc_transcode


def luts():
    with open(os.path.join(GOLDEN, "luts.json")) as f:
        return json.load(f)


def test_lut_tables_match_reference_header_and_derivation():
    L = luts()
    assert o.CODE_LUT.reshape(-1).tolist() == L["code_lut"]
    assert o.CODE_LUT.reshape(-1).tolist() == L["header"]["NVFP4_MXFP6_CODE_LUT"]
    assert o.BUMP_LUT.tolist() == L["bump_lut"] == L["header"]["NVFP4_MXFP6_BUMP_LUT"]
    assert o.SUB_MANT_BITS.tolist() == L["sub_mant_bits"] == L["header"]["NVFP4_MXFP6_SUB_MANT_BITS"]
    assert o.SUB_EXP.tolist() == L["sub_exp"] == L["header"]["NVFP4_MXFP6_SUB_EXP"]
    assert o.E2M3_POS.tolist() == L["e2m3_pos"]
    assert o.E4M3.value.tolist() == L["e4m3_book_value"]


def test_pair_lut_matches_reference_rounding():
    assert o.PAIR_LUT.reshape(-1).tolist() == luts()["pair_lut"]
    # d == 0 is the reference CODE_LUT
    assert np.array_equal(o.PAIR_LUT[:, 0, :], o.CODE_LUT)


def test_cuda_header_tables_match_oracle():
    """The tables compiled into the CUDA library equal the oracle's."""
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    txt = open(os.path.join(root, "bitdance_b200", "csrc", "transcode_lut.cuh")).read()

    def arr(name):
        m = re.search(name + r"\[\d+\] = \{([^}]*)\}", txt)
        return np.array([int(x.strip().rstrip("u"), 0) for x in m.group(1).split(",")])

    assert np.array_equal(arr("kCodeLut").reshape(8, 8), o.CODE_LUT)
    assert np.array_equal(arr("kBumpLut"), o.BUMP_LUT)
    assert np.array_equal(arr("kSubMantBits"), o.SUB_MANT_BITS)
    assert np.array_equal(arr("kSubExp"), o.SUB_EXP)
    assert np.array_equal(arr("kPairLut").reshape(8, 8, 8), o.PAIR_LUT)
    # E4M3 container bytes decode to the same values as the E2M3 codes
    e4 = arr("kE2M3ToE4M3")
    for i, b in enumerate(e4):
        e, m = (b >> 3) & 15, b & 7
        val = 0.0 if b == 0 else (1 + m / 8) * 2.0 ** (e - 7)
        assert val == o.E2M3_POS[i]
    # permute words hold the pair table bytes
    p6 = arr("kPermE2M3").astype(np.uint64)
    p8 = arr("kPermE4M3").astype(np.uint64)
    for cls in range(64):
        mb, d = divmod(cls, 8)
        w6 = [(int(p6[2 * cls + (g >> 2)]) >> (8 * (g & 3))) & 0xFF for g in range(8)]
        w8 = [(int(p8[2 * cls + (g >> 2)]) >> (8 * (g & 3))) & 0xFF for g in range(8)]
        assert w6 == o.PAIR_LUT[mb, d].tolist()
        assert w8 == [int(e4[c]) for c in o.PAIR_LUT[mb, d]]


def test_testvec_1234_golden_mxfp6():
    """kernel/nvfp4_codec.py write_testvec(4096, seed=1234): decode the reference's bytes."""
    g = golden("testvec_1234.npz")
    codes = g["codes"].reshape(-1, 32)
    e8, e6 = o.golden_mxfp6(g["scales"], codes)
    assert np.array_equal(e8, g["golden_e8m0"])
    assert np.array_equal(e6.reshape(-1), g["golden_e2m3"])
    # the per-16 pair rule with equal halves is the per-32 rule
    e8p, e6p = o.transcode_pair16(np.repeat(g["scales"], 2), codes)
    assert np.array_equal(e8p, e8) and np.array_equal(e6p, e6)


def test_testvec_1234_regenerated_inputs():
    """Re-running the reference's generator through the oracle's encoder gives its bytes."""
    g = golden("testvec_1234.npz")
    rng = np.random.default_rng(1234)
    n = 4096 * 32
    x = np.concatenate([rng.normal(0.0, 120.0, n // 2), rng.uniform(-500.0, 500.0, n - n // 2)])
    rng.shuffle(x)
    sb, cc = o.encode_nvfp4(x)
    assert np.array_equal(sb, g["scales"])
    assert np.array_equal(cc.reshape(-1), g["codes"])


@pytest.mark.parametrize("i", range(4))
def test_selftest_tensors(i):
    """nvfp4_codec.selftest tensors: encode, transcode and the float emulation."""
    g = golden("selftest_subset.npz")
    x = g[f"x{i}"]
    sb, cc = o.encode_nvfp4(x)
    assert np.array_equal(sb, g[f"scale{i}"])
    assert np.array_equal(cc, g[f"codes{i}"])
    e8, e6 = o.golden_mxfp6(sb, cc)
    assert np.array_equal(e8, g[f"e8m0_{i}"]) and np.array_equal(e6, g[f"e2m3_{i}"])
    deq = o.dequant_mxfp6(e8, e6).reshape(-1)
    assert np.array_equal(deq, g[f"deq{i}"])
    assert np.array_equal(o.storage_to_mxfp6_revised(x), g[f"deq{i}"])


def test_encode_per16_two_level_scale():
    g = golden("encode16.npz")
    codes, sb, s_t = o.quantize_b_nvfp4(g["w"], block=16)
    assert np.float32(s_t) == g["s_t"][0]
    assert np.array_equal(sb.reshape(-1), g["scales"])
    assert np.array_equal(codes.reshape(-1, 16), g["codes"])


def test_activation_mxfp6_quantiser():
    g = golden("amxfp6.npz")
    codes, e8 = o.quantize_a_mxfp6(g["x"])
    assert np.array_equal(e8.reshape(-1).astype(np.int64) - 127, g["exp"])
    val = np.where((codes >> 5) & 1, -1.0, 1.0) * o.E2M3_POS[codes & 31]
    assert np.array_equal(np.abs(val), np.abs(g["data"]))
    assert np.array_equal(val[g["data"] != 0], g["data"][g["data"] != 0])
    deq = o.dequant_operand(codes, e8)
    assert np.array_equal(np.abs(deq), np.abs(g["deq"]))


def test_pair_rule_matches_reference_primitives():
    g = golden("pair16.npz")
    e8, e6 = o.transcode_pair16(g["scales"], g["codes"])
    assert np.array_equal(e8, g["e8m0"])
    assert np.array_equal(e6, g["e2m3"])


def test_c_oracle_matches_numpy_oracle(orc):
    g = golden("pair16.npz")
    packed = o.pack_nibbles(g["codes"])
    e6, e8 = orc_transcode(orc, packed, g["scales"], 16)
    assert np.array_equal(e8, g["e8m0"])
    assert np.array_equal(e6.reshape(-1, 32), g["e2m3"])
    t = golden("testvec_1234.npz")
    e6, e8 = orc_transcode(orc, o.pack_nibbles(t["codes"].reshape(-1, 32)), t["scales"], 32)
    assert np.array_equal(e8, t["golden_e8m0"]) and np.array_equal(e6, t["golden_e2m3"])


def test_c_oracle_tables(orc):
    code = np.zeros(64, np.uint8)
    bump = np.zeros(8, np.uint8)
    pair = np.zeros(512, np.uint8)
    orc.orc_tables(code.ctypes.data, bump.ctypes.data, pair.ctypes.data)
    assert np.array_equal(code.reshape(8, 8), o.CODE_LUT)
    assert np.array_equal(pair.reshape(8, 8, 8), o.PAIR_LUT)


def test_sweep_generator_covers_relative_exponents():
    packed, sc = o.gen_transcode_sweep(20000, seed=5)
    mb, ex = o.decode_e4m3_byte(sc.reshape(-1, 2))
    e = ex + o.BUMP_LUT[mb]
    d = np.abs(e[:, 0] - e[:, 1])
    assert set(range(8)).issubset(set(d.tolist()))
    assert ((sc >> 3) == 0).any()          # subnormal scale bytes present
    codes = o.unpack_nibbles(packed).reshape(-1, 32)
    assert ((codes[:, :16] & 7) == 0).all(axis=1).any()   # zero-data 16-blocks present


def test_oracle_rejects_non_finite():
    with pytest.raises(ValueError):
        o.quantize_a_mxfp6(np.array([[np.nan] + [0.0] * 31], np.float32))


def test_gemm_gold_small_known_answer():
    """verify_w4a6.py's constant-operand identity C = K * a * b * b_scale
    (kernel/verify_w4a6.py:122-193), through the oracle's dequant path."""
    M, N, K = 4, 8, 256
    a_codes = np.full((M, K), 0x15, np.uint8)        # E2M3 0b010101 = +3.25
    a_e8 = np.full((M, K // 32), 127, np.uint8)
    b = np.full((N, K), o.E2M1_POS.tolist().index(2.0), np.uint8)
    sc = np.full((N, K // 16), 0x38, np.uint8)       # E4M3 1.0
    e6, e8 = o.transcode_b(o.pack_nibbles(b), sc, 16)
    C = o.gemm_gold(a_codes, a_e8, e6, e8, 1.0)
    assert np.all(C == K * 3.25 * 2.0)
