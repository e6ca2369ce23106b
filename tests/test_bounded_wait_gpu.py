"""Failure detection without a GPU fault: a wait that nothing will satisfy ends as a status
the host reads, and the context stays usable. The diagnostic kernel waits, with a short limit
(about 1 ms), on an mbarrier that nothing arrives at, through the same bounded mbar_wait that
every role of the GEMM uses; a second warp waiting with the GEMM's default limit leaves
through the abort flag the first one raises."""
import ctypes

import numpy as np
import pytest

import w4a6_oracle as o


def test_selftest_rejects_bad_limits():
    from bitdance_b200 import build
    build.build_library()
    from bitdance_b200 import _lib
    lib = _lib.load()
    assert lib.bd_selftest_bounded_wait(10, None) == _lib.BD_ERR_INVALID_ARG
    assert lib.bd_selftest_bounded_wait(1 << 40, None) == _lib.BD_ERR_INVALID_ARG


@pytest.mark.gpu
def test_wait_that_runs_out_reports_and_context_survives():
    import torch
    import bitdance_b200 as bd
    from bitdance_b200 import _lib, ops
    word = ops.selftest_bounded_wait(2_000_000)
    assert word == _lib.BD_DEVERR_WAIT_TMA
    assert bd.device_error() == 0  # cleared by the read
    # the context is intact: a GEMM right after is correct and leaves no error
    M, N, K = 8, 256, 512
    rng = np.random.default_rng(9)
    a_codes, a_e8 = o.quantize_a_mxfp6(rng.standard_normal((M, K)).astype(np.float32))
    b_codes, b_sc, s_t = o.quantize_b_nvfp4((rng.standard_normal((N, K)) * 0.02)
                                            .astype(np.float32), block=16)
    b_packed = o.pack_nibbles(b_codes)
    acts = bd.pack_activations(torch.from_numpy(a_codes).cuda(), torch.from_numpy(a_e8).cuda())
    wts = bd.pack_weights(torch.from_numpy(b_packed).cuda(), torch.from_numpy(b_sc).cuda(),
                          float(s_t))
    C = bd.w4a6_gemm(acts, wts).float().cpu().numpy()
    e6, e8 = o.transcode_b(b_packed, b_sc, 16)
    assert o.rel_linf(o.gemm_gold(a_codes, a_e8, e6, e8, float(s_t)), C) <= 1e-2
    assert bd.device_error() == 0
