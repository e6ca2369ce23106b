"""NVFP4 -> MXFP6 transcode on the GPU, bit-exact against the reference's golden vectors and
the CPU oracle (per-32 rule of kernel/nvfp4_codec.py:66-76 and the per-16 pair rule)."""
import numpy as np
import pytest

import w4a6_oracle as o
from conftest import golden, orc_transcode

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def gpu_transcode(packed, scales, scale_block=16):
    from bitdance_b200 import transcode
    e6, e8 = transcode(dev(np.asarray(packed, np.uint8).reshape(-1)),
                       dev(np.asarray(scales, np.uint8).reshape(-1)), scale_block)
    torch.cuda.synchronize()
    return e6.cpu().numpy(), e8.cpu().numpy()


def test_reference_testvec_1234_per32():
    """kernel/nvfp4_codec.py `gen` vector (4096 blocks, seed 1234) -> `verify` byte-for-byte."""
    g = golden("testvec_1234.npz")
    e6, e8 = gpu_transcode(o.pack_nibbles(g["codes"].reshape(-1, 32)), g["scales"], 32)
    assert np.array_equal(e8, g["golden_e8m0"])
    assert np.array_equal(e6, g["golden_e2m3"])


def test_reference_testvec_as_per16_pairs():
    g = golden("testvec_1234.npz")
    e6, e8 = gpu_transcode(o.pack_nibbles(g["codes"].reshape(-1, 32)),
                           np.repeat(g["scales"], 2), 16)
    assert np.array_equal(e8, g["golden_e8m0"])
    assert np.array_equal(e6, g["golden_e2m3"])


@pytest.mark.parametrize("i", range(4))
def test_reference_selftest_tensors(i):
    g = golden("selftest_subset.npz")
    e6, e8 = gpu_transcode(o.pack_nibbles(g[f"codes{i}"]), g[f"scale{i}"], 32)
    assert np.array_equal(e8, g[f"e8m0_{i}"])
    assert np.array_equal(e6.reshape(-1, 32), g[f"e2m3_{i}"])
    assert np.array_equal(o.dequant_mxfp6(e8, e6.reshape(-1, 32)).reshape(-1), g[f"deq{i}"])


def test_pair_rule_golden():
    g = golden("pair16.npz")
    e6, e8 = gpu_transcode(o.pack_nibbles(g["codes"]), g["scales"], 16)
    assert np.array_equal(e8, g["e8m0"])
    assert np.array_equal(e6.reshape(-1, 32), g["e2m3"])


def test_every_scale_byte_pair(orc):
    """All 65536 (s0, s1) byte pairs -- sign bits, subnormals, zero and NaN bytes included."""
    s = np.arange(65536, dtype=np.uint32)
    scales = np.stack([s & 0xFF, s >> 8], 1).astype(np.uint8)
    codes = np.random.default_rng(3).integers(0, 256, (65536, 16), dtype=np.uint8)
    e6, e8 = gpu_transcode(codes, scales, 16)
    r6, r8 = orc_transcode(orc, codes, scales, 16)
    assert np.array_equal(e8, r8)
    assert np.array_equal(e6, r6)


@pytest.mark.parametrize("nblk", [1, 3, 255, 257, 100003])
def test_ragged_sizes(orc, nblk):
    packed, sc = o.gen_transcode_sweep(nblk, seed=nblk)
    e6, e8 = gpu_transcode(packed, sc, 16)
    r6, r8 = orc_transcode(orc, packed, sc, 16)
    assert np.array_equal(e8, r8) and np.array_equal(e6, r6)


def test_empty_input_is_a_noop():
    from bitdance_b200 import _lib
    assert _lib.load().bd_transcode_nvfp4_to_mxfp6(None, None, None, None, 0, 16, None) == 0


def test_misaligned_output_is_rejected():
    from bitdance_b200 import BitdanceError, transcode
    codes = torch.zeros(32, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(4, dtype=torch.uint8, device="cuda")
    out = torch.zeros(80, dtype=torch.uint8, device="cuda")
    with pytest.raises(BitdanceError):
        transcode(codes, sc, 16, e2m3=out[1:65])


def test_config5_one_gib(orc):
    """Config 5 at full size: 1 GiB of packed codes (2^31 codes) in one launch, every byte of
    the output compared with the C oracle, chunk by chunk."""
    chunk = 1 << 22                      # blocks per chunk (64 MiB of codes)
    nchunks = 16                         # 16 x 64 MiB = 1 GiB
    nblk = chunk * nchunks
    codes = torch.empty(nblk * 16, dtype=torch.uint8, device="cuda")
    scales = torch.empty(nblk * 2, dtype=torch.uint8, device="cuda")
    host = []
    for j in range(nchunks):
        p, s = o.gen_transcode_sweep(chunk, seed=1000 + j)
        codes[j * chunk * 16:(j + 1) * chunk * 16].copy_(torch.from_numpy(p))
        scales[j * chunk * 2:(j + 1) * chunk * 2].copy_(torch.from_numpy(s))
        host.append((p, s))
    from bitdance_b200 import transcode
    e6, e8 = transcode(codes, scales, 16)
    torch.cuda.synchronize()
    for j, (p, s) in enumerate(host):
        r6, r8 = orc_transcode(orc, p, s, 16, nthreads=16)
        assert np.array_equal(e8[j * chunk:(j + 1) * chunk].cpu().numpy(), r8)
        assert np.array_equal(e6[j * chunk * 32:(j + 1) * chunk * 32].cpu().numpy(), r6)
