"""The C-ABI library: it loads, exports every entry point include/bitdance_b200.h declares,
and rejects bad arguments before touching a device (no compute calls here). CPU only."""
import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "bitdance_b200.h")


def declared_functions():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(bd_[a-z0-9_]+)\s*\(", txt)))


@pytest.fixture(scope="module")
def lib():
    from bitdance_b200 import build
    build.build_library()
    from bitdance_b200 import _lib
    return _lib.load()


def test_header_declares_the_entry_points():
    fns = declared_functions()
    for f in ("bd_transcode_nvfp4_to_mxfp6", "bd_w4a6_gemm", "bd_w4a6_gemm_ex",
              "bd_splitk_reduce", "bd_pack_b", "bd_pack_b_e4m3", "bd_pack_a", "bd_query_workspace"):
        assert f in fns


def test_library_exports_every_declared_symbol(lib):
    from bitdance_b200 import _lib
    for f in declared_functions():
        assert hasattr(lib, f), f"{f} missing from libbitdance_b200.so"
        assert f in _lib.SIGNATURES, f"{f} has no ctypes signature"


def test_version_and_status_text(lib):
    assert lib.bd_version() >= 100
    assert lib.bd_status_string(0) == b"ok"
    assert b"shape" in lib.bd_status_string(-2)


def test_gemm_rejects_bad_arguments_before_launch(lib):
    P = ctypes.c_void_p
    ok = P(4096)  # never dereferenced: validation fails first
    g = lib.bd_w4a6_gemm
    # null pointer
    assert g(None, ok, ok, ok, ok, 1.0, None, 16, 128, 128, 1, 0, 0, 0, None, 0, None) == -1
    # bad out dtype / epilogue / split mode
    assert g(ok, ok, ok, ok, ok, 1.0, None, 16, 128, 128, 1, 0, 7, 0, None, 0, None) == -1
    assert g(ok, ok, ok, ok, ok, 1.0, None, 16, 128, 128, 1, 0, 0, 9, None, 0, None) == -1
    assert g(ok, ok, ok, ok, ok, 1.0, None, 16, 128, 128, 1, 5, 0, 0, None, 0, None) == -1
    # bias epilogue without bias
    assert g(ok, ok, ok, ok, ok, 1.0, None, 16, 128, 128, 1, 0, 0, 1, None, 0, None) == -1
    # shapes: N % 128, K % 128, M <= 0
    assert g(ok, ok, ok, ok, ok, 1.0, None, 16, 100, 128, 1, 0, 0, 0, None, 0, None) == -2
    assert g(ok, ok, ok, ok, ok, 1.0, None, 16, 128, 96, 1, 0, 0, 0, None, 0, None) == -2
    assert g(ok, ok, ok, ok, ok, 1.0, None, 0, 128, 128, 1, 0, 0, 0, None, 0, None) == -2
    # misaligned operand
    assert g(ok, P(4097), ok, ok, ok, 1.0, None, 16, 128, 128, 1, 0, 0, 0, None, 0, None) == -3


def test_gemm_ex_validates_flags_then_arguments(lib):
    P = ctypes.c_void_p
    ok = P(4096)
    g = lib.bd_w4a6_gemm_ex
    # unknown flag bit
    assert g(ok, ok, ok, ok, ok, 1.0, None, 16, 128, 128, 1, 0, 0, 0, None, 0, 16, None) == -1
    # known flags (BD_GEMM_B_E4M3 = 4, BD_GEMM_SINGLE_CTA = 8 among them), then the same checks
    # as bd_w4a6_gemm
    assert g(None, ok, ok, ok, ok, 1.0, None, 16, 128, 128, 1, 0, 0, 0, None, 0, 15, None) == -1
    assert g(ok, ok, ok, ok, ok, 1.0, None, 16, 100, 128, 1, 0, 0, 0, None, 0, 1, None) == -2


def test_probe_and_scale_conversion_reject_bad_arguments(lib):
    assert lib.bd_probe_mma_peak(0, 256, 0, None) == -1
    assert lib.bd_probe_mma_peak(1 << 22, 256, 0, None) == -1
    assert lib.bd_probe_mma_peak(1024, 24, 0, None) == -1
    assert lib.bd_probe_mma_peak(1024, 272, 1, None) == -1
    assert lib.bd_probe_mma_peak(1024, 128, 2, None) == -1  # the pair form is N = 256 only
    assert lib.bd_probe_mma_peak(1024, 256, 3, None) == -1
    assert lib.bd_scales_e8m0_to_e4m3_pairs(None, None, -1, None) == -2
    assert lib.bd_scales_e8m0_to_e4m3_pairs(None, None, 0, None) == 0
    assert lib.bd_scales_e8m0_to_e4m3_pairs(None, None, 16, None) == -1
    assert lib.bd_scales_e8m0_to_e4m3_pairs(8, 9, 16, None) == -3


def test_transcode_rejects_bad_arguments(lib):
    P = ctypes.c_void_p
    ok = P(4096)
    t = lib.bd_transcode_nvfp4_to_mxfp6
    assert t(ok, ok, ok, ok, 8, 24, None) == -1      # scale_block
    assert t(ok, ok, ok, ok, -1, 16, None) == -2     # negative size
    assert t(ok, ok, ok, ok, 0, 16, None) == 0       # empty input is a no-op
    assert t(None, ok, ok, ok, 8, 16, None) == -1
    assert t(P(4100), ok, ok, ok, 8, 16, None) == -3
    assert t(ok, P(4097), ok, ok, 8, 16, None) == -3  # per-16 scales read as u16


def test_pack_rejects_bad_shapes(lib):
    P = ctypes.c_void_p
    ok = P(4096)
    assert lib.bd_pack_b(ok, ok, ok, ok, 100, 128, None) == -2
    assert lib.bd_pack_b_e4m3(ok, ok, ok, ok, 100, 128, None) == -2
    assert lib.bd_pack_a(ok, ok, ok, ok, 4, 100, None) == -2
    assert lib.bd_splitk_reduce(ok, ok, None, 1.0, 4, 6, 2, 0, 0, None) == -2


def test_workspace_query(lib):
    assert lib.bd_query_workspace(64, 1024, 1024, 4, 0) == 4 * 64 * 1024 * 4
    assert lib.bd_query_workspace(64, 1024, 1024, 4, 1) == 0   # planes need none
    assert lib.bd_query_workspace(64, 1024, 1024, 1, 0) == 0
    assert lib.bd_query_workspace(64, 1000, 1024, 4, 0) == 0   # invalid shape
    # stream-K (split_k 0): slots for (grid x 2) partial tiles of 16 token rows x 256 weight
    # rows + one counter per tile; with no device visible the library assumes 148 SMs
    tiles = 14336 // 256
    slots = 148 * 2 * 16 * 256 * 4
    assert lib.bd_query_workspace(16, 14336, 4096, 0, 0) == slots + (tiles * 4 + 255) // 256 * 256
    # a small problem: grid = units = tiles x K/128 chunks
    tiles, units = 2 * 1, 2 * 1 * 4
    assert lib.bd_query_workspace(100, 384, 512, 0, 0) == \
        units * 2 * 128 * 256 * 4 + (tiles * 4 + 255) // 256 * 256


def test_psg_shim_validation_matches_reference_errors():
    from bitdance_b200.psg import compile_preshuffle_gemm_a8 as c
    with pytest.raises(ValueError):
        c(K=256, tile_m=128, tile_n=128, tile_k=128, in_dtype="nope")
    with pytest.raises(NotImplementedError):
        c(K=256, tile_m=128, tile_n=128, tile_k=128, in_dtype="fp8")
    with pytest.raises(ValueError):
        c(K=256, tile_m=128, tile_n=128, tile_k=128, in_dtype="w4a6_tc", out_dtype="fp32")
    with pytest.raises(NotImplementedError):
        c(K=256, tile_m=128, tile_n=128, tile_k=256, in_dtype="w4a6_tc")
    with pytest.raises(ValueError):
        c(K=256, tile_m=128, tile_n=128, tile_k=128, in_dtype="w4a6_tc", split_k=0)
    with pytest.raises(ValueError):
        c(K=384, tile_m=128, tile_n=128, tile_k=128, in_dtype="w4a6_tc", split_k=2)
    with pytest.raises(ValueError):
        c(K=256, tile_m=128, tile_n=128, tile_k=128, in_dtype="w4a6_tc", split_reduce="tree")
    with pytest.raises(ValueError):
        c(K=256, tile_m=128, tile_n=128, tile_k=128, in_dtype="w4a6_tc", split_reduce="atomic",
          epilogue="bias")
    with pytest.raises(NotImplementedError):
        c(K=256, tile_m=128, tile_n=128, tile_k=128, in_dtype="w4a6_tc", use_hw_transcode=True)
    # the alias resolves like the reference's (psg:341-342)
    assert c(K=256, tile_m=128, tile_n=128, tile_k=128, in_dtype="w6a6_tc").K == 256
    # the MXFP4-weight arm the reference's verify script cross-checks against (psg:411-423)
    assert c(K=256, tile_m=128, tile_n=128, tile_k=128, in_dtype="w4a6").in_dtype == "w4a6"
    with pytest.raises(NotImplementedError):
        c(K=256, tile_m=128, tile_n=128, tile_k=256, in_dtype="w4a6")


def test_psg_launch_reads_weights_as_the_reference_bytes(monkeypatch):
    """The drop-in launch passes BD_GEMM_B_E4M3: b / scale_b hold the reference's code and E4M3
    scale bytes (only regrouped), so buffers filled the way kernel/verify_w4a6.py and
    kernel/bench_sweep.py fill them mean the same. Checked on the call the shim makes."""
    from bitdance_b200 import _lib, psg
    seen = []
    monkeypatch.setattr(psg, "call", lambda name, *args: seen.append((name, args)))
    launch = psg.compile_preshuffle_gemm_a8(M=16, N=256, K=256, tile_m=128, tile_n=256,
                                            tile_k=128, in_dtype="w4a6_tc", out_dtype="bf16")
    launch(4096, 8192, 12288, 16384, 20480, 24576, 28672, 16, 256, 0, b_tensor_scale=0.5)
    (name, args), = seen
    assert name == "bd_w4a6_gemm_ex"
    assert args[-2] == _lib.BD_GEMM_B_E4M3 and args[5] == 0.5


def test_product_path_never_imports_the_oracle():
    pkg = os.path.join(ROOT, "bitdance_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith(".py"):
                txt = open(os.path.join(dirpath, f)).read()
                assert "w4a6_oracle" not in txt and "oracle/" not in txt and "liborc" not in txt, f
