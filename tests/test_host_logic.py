"""Host-side logic without a GPU: the drop-in module tree, the MXFP4 -> E4M3 scale rule of the
"w4a6" arm checked against the oracle's pair rule, Workspace re-zeroing after a device error,
and the device check of tensor arguments. CPU only."""
import json
import os
import sys
import types

import numpy as np
import pytest

import w4a6_oracle as o
from conftest import GOLDEN, ROOT

DROPIN = os.path.join(ROOT, "bitdance_b200", "dropin")


def e4m3_of_e8m0(e):
    """The mapping bd_scales_e8m0_to_e4m3_pairs applies (restated for the check)."""
    s = int(e) - 127
    if -6 <= s <= 8:
        return (s + 7) << 3
    if -9 <= s <= -7:
        return 0x04 >> (-7 - s)
    return None


def test_mxfp4_scales_become_exact_nvfp4_pairs():
    """For every E8M0 exponent with an E4M3 form, both 16-blocks scaled by that E4M3 byte go
    through the per-16 pair rule to the MXFP4 block itself: E8M0 unchanged and each E2M3 value
    equal to the E2M1 value (the reference's "w4a6" arm, psg_preshuffle_gemm.py:411-423)."""
    codes = np.tile(np.arange(16, dtype=np.uint8), 2)[None, :]      # every nibble, both halves
    mxfp4 = np.where(codes & 8, -1.0, 1.0) * o.E2M1_POS[codes & 7]
    n_ok = 0
    for e in range(256):
        b = e4m3_of_e8m0(e)
        if b is None:
            assert not (-9 <= e - 127 <= 8)
            continue
        e8, e6 = o.transcode_pair16(np.array([[b, b]], np.uint8), codes)
        assert int(e8[0]) == e
        val = o.dequant_mxfp6(e8, e6) / 2.0 ** (e - 127)
        assert np.array_equal(val, mxfp4), e
        n_ok += 1
    assert n_ok == 18


def test_dropin_modules_resolve_the_reference_imports():
    sys.path.insert(0, DROPIN)
    try:
        import flydsl.compiler as flyc
        import flydsl.expr as fx
        from flydsl.compiler.jit_argument import from_c_void_p
        from kernel.nvfp4_mxfp6_gemm_tiled import build_LUT12
        from psg.preshuffle_gemm import compile_preshuffle_gemm_a8
        import bitdance_b200.psg as bp
        assert compile_preshuffle_gemm_a8 is bp.compile_preshuffle_gemm_a8
        p = from_c_void_p(fx.Int8, 4096)
        assert p.value == 4096 and p.dtype is fx.Int8
        for name in ("Int8", "Int16", "Int32", "Float32", "BFloat16"):
            assert hasattr(fx, name)
        f = lambda *a: a  # noqa: E731
        assert flyc.compile(f, 1, 2) is f
        lut = build_LUT12()
    finally:
        sys.path.remove(DROPIN)
        for m in [m for m in sys.modules if m.split(".")[0] in ("flydsl", "psg", "kernel")]:
            del sys.modules[m]
    # the v31 construction (kernel/hip/w4a6_tc_gemm_v31.hip:668-673) over the reference's
    # CODE_LUT literals (fixture written from kernel/transcode_lut.h)
    code = json.load(open(os.path.join(GOLDEN, "luts.json")))["header"]["NVFP4_MXFP6_CODE_LUT"]
    want = []
    for s in range(8):
        for b in range(256):
            lo, hi = b & 0xF, b >> 4
            cl = (((lo >> 3) & 1) << 5) | code[s * 8 + (lo & 7)]
            ch = (((hi >> 3) & 1) << 5) | code[s * 8 + (hi & 7)]
            want.append((cl & 0x3F) | ((ch & 0x3F) << 6))
    assert lut == want


@pytest.mark.skipif(not os.path.isdir("/root/reference/kernel"), reason="reference checkout absent")
def test_reference_scripts_import_through_the_dropin(monkeypatch):
    """kernel/verify_w4a6.py and kernel/bench_sweep.py import unmodified with the drop-in tree
    on the path (only their imports run; nothing is launched without a GPU)."""
    import importlib.util
    monkeypatch.syspath_prepend(DROPIN)
    try:
        for name in ("verify_w4a6", "bench_sweep"):
            path = os.path.join("/root/reference/kernel", name + ".py")
            spec = importlib.util.spec_from_file_location("_ref_" + name, path)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            assert callable(mod.main)
    finally:
        for m in [m for m in sys.modules if m.split(".")[0] in ("flydsl", "psg", "kernel")]:
            del sys.modules[m]


def test_workspace_rezeroes_after_a_wait_error():
    torch = pytest.importorskip("torch")
    from bitdance_b200 import _lib, ops
    ws = ops.Workspace()
    b = ws.get(1024, "cpu", key=(1, 2, 3))
    b.fill_(7)
    assert int(ws.get(1024, "cpu", key=(1, 2, 3))[:1024].min()) == 7  # same shape: kept
    ops._note_device_error(_lib.BD_DEVERR_NONFINITE)                   # not a wait: kept
    assert int(ws.get(1024, "cpu", key=(1, 2, 3))[:1024].min()) == 7
    ops._note_device_error(_lib.BD_DEVERR_WAIT_TMA)                    # a wait ran out
    assert int(ws.get(1024, "cpu", key=(1, 2, 3))[:1024].count_nonzero()) == 0
    b.fill_(5)
    assert int(ws.get(1024, "cpu", key=(1, 2, 3))[:1024].min()) == 5   # once only
    assert int(ws.get(1024, "cpu", key=(9, 9, 9))[:1024].count_nonzero()) == 0  # new shape
    del torch


def test_tensors_on_another_device_are_refused(monkeypatch):
    torch = pytest.importorskip("torch")
    from bitdance_b200 import ops
    monkeypatch.setattr(torch.cuda, "current_device", lambda: 0)
    ops._check_device(types.SimpleNamespace(device=torch.device("cuda", 0)), "x")
    ops._check_device(types.SimpleNamespace(device=torch.device("cuda")), "x")
    with pytest.raises(ValueError, match="cuda:1"):
        ops._check_device(types.SimpleNamespace(device=torch.device("cuda", 1)), "x")
