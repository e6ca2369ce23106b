"""``build_LUT12()``: the 12-bit transcode table the reference's LUT arm passes to its kernel
(REPRODUCE.md:574-577; the same construction as kernel/hip/w4a6_tc_gemm_v31.hip:668-673).
Entry (mb << 8) | byte holds the E2M3 codes of the byte's two E2M1 nibbles under an E4M3 scale
with mantissa bits mb: low nibble in bits 0..5, high nibble in bits 6..11, each
sign << 5 | CODE_LUT[mb * 8 + magnitude]. This library's GEMM does not read it (its transcode
tables are compiled in); the table is built so scripts that pass it run unchanged."""
import importlib.util
import os

_GEN = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                    "csrc", "gen_transcode_lut.py")


def _code_lut():
    spec = importlib.util.spec_from_file_location("_bd_gen_transcode_lut", _GEN)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    code, _, _, _ = mod.tables()
    return code


def build_LUT12():  # noqa: N802 - the reference's name
    code = _code_lut()
    lut = []
    for mb in range(8):
        for b in range(256):
            lo, hi = b & 0xF, b >> 4
            cl = ((lo >> 3) & 1) << 5 | code[mb * 8 + (lo & 7)]
            ch = ((hi >> 3) & 1) << 5 | code[mb * 8 + (hi & 7)]
            lut.append((cl & 0x3F) | ((ch & 0x3F) << 6))
    return lut
