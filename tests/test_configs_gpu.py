"""The W4A6 GEMM at every BASELINE config's own shapes and distributions, and a bit-exact
read-back of the weights the GEMM transcodes on chip.

Configs: 1 -- M=128, N=K=4096, A ~ N(0,1), B ~ N(0,0.02); 2 -- decode,
N=14336, K=4096, M in {1,4,16,32,64}, Student-t weights, outlier-channel activations;
3 -- prefill M=8192, gate/up 14336x4096 and down 4096x14336, config-2 distributions;
4 -- Llama-3-70B shape N=28672, K=8192, M in {16, 4096}, B ~ N(0,0.015), A ~ N(0,1).
Operands are drawn on the GPU from seeded generators, quantised by the device quantisers (whose
bytes are checked against the oracle on sampled rows), and the GEMM's sampled token rows
(every token tile, all N) are checked against an fp64 dequantise-then-matmul gold at
max-abs-rel <= 1e-2 plus an elementwise bf16 bound (tests/bigshape.py)."""
import numpy as np
import pytest

import w4a6_oracle as o
from bigshape import Acts, Weights, check_rows, gemm_rows, gold_rows

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def run_case(M, N, K, a_kind, b_kind, b_std, seed, **kw):
    import bitdance_b200 as bd
    w = Weights(torch, N, K, b_kind, b_std, seed + 1)
    a = Acts(torch, M, K, a_kind, seed)
    w.check()
    a.check()
    out = bd.w4a6_gemm(a.gemm, w.gemm, **kw)
    torch.cuda.synchronize()
    assert bd.device_error() == 0
    C, Cabs = gold_rows(a, w)
    check_rows(gemm_rows(torch, out, a), C, Cabs)
    return a, w, C, Cabs


def test_config1_full_size_device_quantised():
    run_case(128, 4096, 4096, "normal", "normal", 0.02, seed=10)


@pytest.mark.parametrize("M", [1, 4, 16, 32, 64])
def test_config2_decode_full_n(M):
    run_case(M, 14336, 4096, "outlier", "t", 0.02, seed=20 + M)


@pytest.mark.parametrize("N,K", [(14336, 4096), (4096, 14336)])
def test_config3_prefill(N, K):
    run_case(8192, N, K, "outlier", "t", 0.02, seed=30 + K // 1024)


@pytest.mark.parametrize("M", [16, 4096])
def test_config4_70b_shape(M):
    run_case(M, 28672, 8192, "normal", "normal", 0.015, seed=40 + M)


def test_config2_split_k_and_stream_k_agree():
    """Decode shape through the stream-K default and the explicit split-K reduce (4 and 8
    splits): every schedule within the tolerance and the elementwise bound of the gold."""
    import bitdance_b200 as bd
    a, w, C, Cabs = run_case(16, 14336, 4096, "outlier", "t", 0.02, seed=50)
    for split_k in (4, 8):
        split = bd.w4a6_gemm(a.gemm, w.gemm, split_k=split_k)
        check_rows(gemm_rows(torch, split, a), C, Cabs)


def _one_hot_tokens(M, K):
    a = np.zeros((M, K), np.uint8)
    a[np.arange(M), np.arange(M) % K] = 0x08     # E2M3 code of +1.0
    return a, np.full((M, K // 32), 127, np.uint8)  # E8M0 1.0


@pytest.mark.parametrize("sideband", ["class", "e4m3"])
@pytest.mark.parametrize("K,split_k", [(128, 1), (256, 0), (1024, 0), (1024, 4)])
def test_one_hot_tokens_read_back_the_transcoded_weights(sideband, K, split_k):
    """Token m holds +1.0 at k = m and zeros elsewhere (M = K), so with an fp32 output and a
    tensor scale of 1.0, C[m, n] is the single product 1.0 * B'[n, m], where B' is the MXFP6
    value the GEMM built on chip from weight row n. Every element of C must equal the oracle's
    dequant(transcode(B)) exactly: the in-GEMM transcode is bit-exact in value for every scale
    byte (0x00..0xFF: zero, subnormal, the largest exponents, sign-bit bytes), through both
    weight layouts and the stream-K / split-K schedules."""
    import bitdance_b200 as bd
    M, N = K, 1024
    rng = np.random.default_rng(K + split_k)
    b_packed = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    b_sc = rng.integers(0, 256, (N, K // 16), dtype=np.uint8)
    b_sc[:, 0] = np.arange(N) % 256                 # every scale byte appears
    a_codes, a_e8 = _one_hot_tokens(M, K)
    acts = bd.pack_activations(torch.from_numpy(a_codes).cuda(), torch.from_numpy(a_e8).cuda())
    w = bd.pack_weights(torch.from_numpy(b_packed).cuda(), torch.from_numpy(b_sc).cuda(), 1.0,
                        sideband=sideband)
    C = bd.w4a6_gemm(acts, w, split_k=split_k, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert bd.device_error() == 0
    e6, e8 = o.transcode_b(b_packed, b_sc, 16)
    deq = o.dequant_operand(e6, e8)                 # (N, K) fp64, exact in fp32
    got = C.cpu().numpy().astype(np.float64)        # (M, N) = (K, N)
    assert np.array_equal(got, deq.T), np.argwhere(got != deq.T)[:4]


def test_one_hot_codes_and_scales_bit_exact():
    """The same read-back, turned into codes: C's column n divided by the oracle's E8M0 scale
    of each 32-block is an E2M3 magnitude, and its index in the E2M3 book is the oracle's code
    (the sign from the sign of C for non-zero codes). Scale pairs drawn over the whole normal
    and subnormal E4M3 range, so relative exponents 0..7 and beyond all occur."""
    import bitdance_b200 as bd
    K = M = 256
    N = 256
    rng = np.random.default_rng(7)
    b_packed = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    # scale pairs with every relative exponent 0..7 and every mantissa class
    s0 = rng.integers(0x01, 0x7F, (N, K // 32), dtype=np.uint8)
    s1 = rng.integers(0x01, 0x7F, (N, K // 32), dtype=np.uint8)
    b_sc = np.stack([s0, s1], axis=-1).reshape(N, K // 16)
    a_codes, a_e8 = _one_hot_tokens(M, K)
    acts = bd.pack_activations(torch.from_numpy(a_codes).cuda(), torch.from_numpy(a_e8).cuda())
    w = bd.pack_weights(torch.from_numpy(b_packed).cuda(), torch.from_numpy(b_sc).cuda(), 1.0)
    C = bd.w4a6_gemm(acts, w, split_k=1, out_dtype=torch.float32).cpu().numpy().T  # (N, K)
    e6, e8 = o.transcode_b(b_packed, b_sc, 16)
    scale = np.exp2(e8.astype(np.float64) - 127)                          # (N, K/32)
    mag = np.abs(C.astype(np.float64)) / np.repeat(scale, 32, axis=1)
    idx = np.searchsorted(o.E2M3_POS, mag)
    assert np.array_equal(o.E2M3_POS[idx], mag)           # every value is an E2M3 magnitude
    assert np.array_equal(idx, (e6 & 0x1F).astype(np.int64))
    nz = (e6 & 0x1F) != 0
    assert np.array_equal(np.signbit(C)[nz], ((e6 >> 5) & 1).astype(bool)[nz])
