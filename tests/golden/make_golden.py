#!/usr/bin/env python3
"""Generate the golden fixtures in this directory by running the REFERENCE's own Python code
(scimg/bitdance, read-only at REF_ROOT). Run in the build container only:

    python tests/golden/make_golden.py REF_ROOT     (or REF_ROOT in the environment)

Nothing at test time reads the reference; the tests read the .npz/.json files written here.
Every fixture records which reference function produced it.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REF_ROOT", "")
if not REF or not os.path.isdir(REF):
    sys.exit("usage: make_golden.py REF_ROOT (the reference checkout, read-only)")

# The reference reads these at import (vector_quant_error.py:156-177); pin the defaults.
os.environ["MXFP6_E4M3_SUBNORMAL"] = "0"
os.environ["MXFP6_E4M3_LEGACY_BOOK"] = "0"
sys.path.insert(0, REF)
sys.path.insert(0, os.path.join(REF, "kernel"))

import vector_quant_error as vq  # noqa: E402
from kernel import nvfp4_codec as codec  # noqa: E402
from kernel import transcode_lut as tl  # noqa: E402


def save(name, **arrays):
    np.savez_compressed(os.path.join(HERE, name), **arrays)
    print("wrote", name, {k: v.shape for k, v in arrays.items()})


def header_tables():
    """Literal tables of kernel/transcode_lut.h, parsed as text."""
    import re
    txt = open(os.path.join(REF, "kernel", "transcode_lut.h")).read()
    out = {}
    for name in ("NVFP4_MXFP6_CODE_LUT", "NVFP4_MXFP6_BUMP_LUT", "NVFP4_MXFP6_SUB_MANT_BITS",
                 "NVFP4_MXFP6_SUB_EXP"):
        m = re.search(name + r"\[\d+\] = \{([^}]*)\}", txt)
        out[name] = [int(x) for x in m.group(1).replace("\n", " ").split(",") if x.strip()]
    return out


def pair_rule_ref(scale16: np.ndarray, codes: np.ndarray):
    """The per-16 pair rule evaluated with the reference's own primitives:
    decode_e4m3_byte / BUMP_LUT (kernel/transcode_lut.py) and nearest_codes
    (vector_quant_error.py:255-280). d is NOT clamped here."""
    mb, exp = tl.decode_e4m3_byte(scale16.reshape(-1, 2))
    bump = tl.BUMP_LUT[mb].astype(np.int64)
    e = exp + bump
    emax = e.max(axis=1)
    d = emax[:, None] - e
    m = 1.0 + mb / 8.0
    half = np.repeat(np.arange(2), 16)
    mag = tl.E2M1_POS[(codes & 7).astype(np.int64)]
    val = m[:, half] * mag / np.exp2((bump + d)[:, half].astype(np.float64))
    q = np.abs(vq.nearest_codes(val, vq.E2M3))
    mag5 = np.abs(q[..., None] - tl.E2M3_POS[None, None, :]).argmin(axis=-1)
    sign = (codes >> 3) & 1
    return (emax + 127).astype(np.uint8), ((sign << 5) | mag5).astype(np.uint8)


def main():
    # the project the fixtures come from, not the checkout path of the machine that made them
    meta = {"reference": "scimg/bitdance",
            "env": {"MXFP6_E4M3_SUBNORMAL": "0", "MXFP6_E4M3_LEGACY_BOOK": "0"}}

    # 1. LUTs: derived by transcode_lut.build_luts and the literal header.
    hdr = header_tables()
    pair_lut = np.zeros((8, 8, 8), np.uint8)
    for mb in range(8):
        m = 1.0 + mb / 8.0
        b = int(tl.BUMP_LUT[mb])
        for d in range(8):
            vals = m * tl.E2M1_POS / 2.0 ** (b + d)
            q = np.abs(vq.nearest_codes(vals[None, :], vq.E2M3))[0]
            pair_lut[mb, d] = np.abs(q[:, None] - tl.E2M3_POS[None, :]).argmin(axis=-1)
    luts = {
        "code_lut": tl.CODE_LUT.reshape(-1).tolist(),
        "bump_lut": tl.BUMP_LUT.tolist(),
        "sub_mant_bits": tl.SUB_MANT_BITS.tolist(),
        "sub_exp": tl.SUB_EXP.tolist(),
        "header": hdr,
        "pair_lut": pair_lut.reshape(-1).tolist(),
        "e2m3_pos": tl.E2M3_POS.tolist(),
        "e4m3_book_value": vq.E4M3.value.tolist(),
        "source": "kernel/transcode_lut.py build_luts; kernel/transcode_lut.h; "
                  "pair_lut via vector_quant_error.nearest_codes",
        **meta,
    }
    with open(os.path.join(HERE, "luts.json"), "w") as f:
        json.dump(luts, f)
    print("wrote luts.json")

    # 2. The reference's binary test vector: nvfp4_codec.write_testvec(n_blocks=4096, seed=1234).
    with tempfile.TemporaryDirectory() as td:
        codec.write_testvec(td, n_blocks=4096, seed=1234)
        rd = lambda n: np.fromfile(os.path.join(td, n), dtype=np.uint8)  # noqa: E731
        save("testvec_1234.npz", scales=rd("scales.bin"), codes=rd("codes.bin"),
             golden_e8m0=rd("golden_e8m0.bin"), golden_e2m3=rd("golden_e2m3.bin"))

    # 3. selftest tensors (nvfp4_codec.selftest, seed vq.SEED): first 4096 elements of each.
    rng = np.random.default_rng(vq.SEED)
    st = {}
    for i, (name, gen) in enumerate(vq.TENSORS):
        x = gen(rng).astype(np.float64, copy=False)[:4096]
        sb, cc, _ = codec.encode_nvfp4(x)
        e8, e6 = codec.golden_mxfp6(sb, cc)
        st[f"x{i}"] = x
        st[f"scale{i}"] = sb
        st[f"codes{i}"] = cc
        st[f"e8m0_{i}"] = e8
        st[f"e2m3_{i}"] = e6
        st[f"deq{i}"] = vq.storage_to_mxfp6(x, vq.E4M3, "revised")
    save("selftest_subset.npz", **st)

    # 4. Per-16 NVFP4 with the two-level scale (remote/quant_real_weights.py:273-287), on a
    #    small N(0, 0.02) matrix; encode with the reference's encode_nvfp4(block=16).
    w = (np.random.default_rng(11).standard_normal((64, 256)) * 0.02).astype(np.float32)
    amax = float(np.max(np.abs(w)))
    s_t = amax / (float(np.max(vq.E4M3.value)) * 6.0)
    scaled = w / np.float32(s_t)
    sb16, c16, _ = codec.encode_nvfp4(scaled.reshape(-1), block=16)
    save("encode16.npz", w=w, s_t=np.array([np.float32(s_t)]), scales=sb16, codes=c16)

    # 5. Direct MXFP6 activations: vq.quantize(x, E8M0, E2M3) (vector_quant_error.py:305, :389).
    xa = np.random.default_rng(12).standard_normal((16, 256)).astype(np.float32)
    xa[:, 7] *= 20.0
    qa = vq.quantize(xa.reshape(-1), vq.E8M0, vq.E2M3)
    save("amxfp6.npz", x=xa, data=qa.data.reshape(16, 256), exp=qa.exp.astype(np.int64),
         deq=qa.deq.reshape(16, 256))

    # 6. Per-16 pair rule on config-5 style inputs, evaluated with reference primitives.
    rng = np.random.default_rng(5)
    nb = 4096
    codes = rng.integers(0, 16, (nb, 32), dtype=np.uint8)
    s0 = rng.integers(0x01, 0x7F, nb, dtype=np.uint8)
    e1 = np.clip(((s0 >> 3) & 0xF).astype(np.int64) + rng.integers(-9, 10, nb), 0, 15)
    s1 = ((e1 << 3) | rng.integers(0, 8, nb)).astype(np.uint8)
    s1 = np.where(s1 == 0x7F, 0x7E, np.where(s1 == 0, 1, s1)).astype(np.uint8)
    same = rng.random(nb) < 0.1
    s1[same] = s0[same]
    sc = np.stack([s0, s1], 1)
    e8, e6 = pair_rule_ref(sc, codes)
    g8, g6 = codec.golden_mxfp6(s0[same], codes[same])
    assert np.array_equal(g8, e8[same]) and np.array_equal(g6, e6[same])
    save("pair16.npz", scales=sc.reshape(-1), codes=codes, e8m0=e8, e2m3=e6)


if __name__ == "__main__":
    main()
