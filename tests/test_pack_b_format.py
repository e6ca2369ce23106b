"""The GEMM's tiled weight layout carries the weight-only parts of the transcode, prepared by
bd_pack_b (pack_b_kernel, bitdance_b200/csrc/transcode.cuh): sign bits moved inside each
32-bit code word, and one 16-bit class word per 32-block instead of its two E4M3 scale bytes.

The packer's two encodings and the GEMM's decode of them (gemm.cuh: nib8_to_e4m3 and the
class-word decode in the transcode loop) are restated here in numpy and checked against the
oracle's per-16 pair rule (transcode_pair16, which follows kernel/nvfp4_codec.py and
kernel/transcode_lut.py): for every pair of scale bytes the decoded magnitude-table rows and
E8M0 byte are the rule's, and every code keeps its sign and magnitude. CPU only; the GPU GEMM
tests check the CUDA code end to end."""
import numpy as np

import w4a6_oracle as o


def scale_class(byte):
    """Info-table class of an E4M3 scale byte: (e + 16) << 3 | mb, e = exponent + bump."""
    mb, exp = o.decode_e4m3_byte(np.asarray(byte, np.int64) & 0x7F)
    e = exp + o.BUMP_LUT[mb].astype(np.int64)
    return ((e + 16) << 3) | mb


def pair_sideband(c0, c1):
    """Packer: class word of a 32-block from its two scale-byte classes."""
    e0, e1 = c0 >> 3, c1 >> 3
    first_big = (e0 > e1).astype(np.int64)
    em = np.where(first_big == 1, e0, e1)
    es = np.where(first_big == 1, e1, e0)
    d = np.minimum(em - es, 7)
    small_row = d * 8 + np.where(first_big == 1, c1, c0) % 8
    big_mb = np.where(first_big == 1, c0, c1) % 8
    return small_row | (big_mb << 6) | (first_big << 9) | ((em - 7) << 10)


def decode_sideband(f):
    """GEMM: table rows (d*8 + mb) of the two 16-blocks and the E8M0 byte."""
    off_small, off_big = (f << 6) & 0xFC0, f & 0x1C0   # rows x 64 (8-copy table)
    first_big = (f & 0x200) != 0
    row0 = np.where(first_big, off_big, off_small) // 64
    row1 = np.where(first_big, off_small, off_big) // 64
    return row0, row1, ((f >> 10) & 0x1F) + 118


def sign_spread(w):
    w = np.asarray(w, np.uint64)
    r = w & 0x77777777
    for i in range(8):
        r |= ((w >> (4 * i + 3)) & 1) << (8 * i + 7 if i < 4 else 8 * (i - 4) + 3)
    return r


def test_class_words_give_the_pair_rule_for_every_scale_pair():
    s = np.arange(256)
    s0, s1 = np.meshgrid(s, s, indexing="ij")
    s0, s1 = s0.ravel(), s1.ravel()
    f = pair_sideband(scale_class(s0), scale_class(s1))
    assert f.max() < 1 << 15
    row0, row1, e8 = decode_sideband(f)
    # the rule: per 16-block (mb, e), emax, d = min(emax - e, 7), E8M0 = emax + 127
    mb, exp = o.decode_e4m3_byte(np.stack([s0, s1], 1))
    e = exp + o.BUMP_LUT[mb].astype(np.int64)
    emax = e.max(axis=1)
    d = np.minimum(emax[:, None] - e, 7)
    assert np.array_equal(row0, d[:, 0] * 8 + mb[:, 0])
    assert np.array_equal(row1, d[:, 1] * 8 + mb[:, 1])
    assert np.array_equal(e8, emax + 127)
    # and the oracle's transcode of a block with those scales uses exactly these rows
    codes = np.random.default_rng(0).integers(0, 16, (s0.size, 32))
    e8_o, e2m3 = o.transcode_pair16(np.stack([s0, s1], 1), codes)
    assert np.array_equal(e8, e8_o.astype(np.int64))
    mags = np.concatenate([o.PAIR_LUT[row0 % 8, row0 // 8][np.arange(s0.size)[:, None], codes[:, :16] & 7],
                           o.PAIR_LUT[row1 % 8, row1 // 8][np.arange(s0.size)[:, None], codes[:, 16:] & 7]],
                          axis=1)
    assert np.array_equal(mags, e2m3 & 0x1F)


def test_moved_sign_bits_reach_their_output_bytes():
    w = np.random.default_rng(1).integers(0, 1 << 32, 4096, dtype=np.uint64)
    p = sign_spread(w)
    m = p & 0x77777777
    sign_lo = p & 0x80808080                      # bytes 0..3 <- elements 0..3
    sign_hi = (p << 4) & 0x80808080               # bytes 0..3 <- elements 4..7
    for i in range(8):
        assert np.array_equal((m >> (4 * i)) & 7, (w >> (4 * i)) & 7)
        src = sign_lo if i < 4 else sign_hi
        assert np.array_equal((src >> (8 * (i % 4) + 7)) & 1, (w >> (4 * i + 3)) & 1)
