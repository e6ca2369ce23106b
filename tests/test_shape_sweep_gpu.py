"""Shape sweep of the W4A6 GEMM (the transcode-isolation config's GEMM sweep): all 64
combinations of M, N, K in {256, 1024, 4096, 8192}, with the first config's operand
distributions (A ~ N(0,1) -> MXFP6, B ~ N(0, 0.02) -> NVFP4 per-16 + fp32 tensor scale),
library-chosen schedule. Operands are drawn on the GPU from seeded generators and quantised by
the device quantisers (their bytes checked against the oracle on sampled rows, once per
operand); the GEMM's sampled token rows (the first and last of every 128-row token tile, all
N) are checked against an fp64 dequantise-then-matmul gold at max-abs-rel <= 1e-2 plus the
elementwise bf16 bound. Operands are cached per (M, K) and (N, K), so each is made once."""
import functools
import itertools

import pytest

from bigshape import Acts, Weights, check_rows, gemm_rows, gold_rows

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SIZES = (256, 1024, 4096, 8192)
CASES = list(itertools.product(SIZES, SIZES, SIZES))


@functools.lru_cache(maxsize=None)
def acts(M, K):
    a = Acts(torch, M, K, "normal", seed=M * 7 + K)
    a.check()
    return a


@functools.lru_cache(maxsize=None)
def weights(N, K):
    w = Weights(torch, N, K, "normal", 0.02, seed=N * 11 + K + 1)
    w.check()
    return w


@pytest.mark.parametrize("M,N,K", CASES)
def test_gemm_shape_sweep(M, N, K):
    import bitdance_b200 as bd
    a, w = acts(M, K), weights(N, K)
    out = bd.w4a6_gemm(a.gemm, w.gemm)
    torch.cuda.synchronize()
    assert bd.device_error() == 0
    C, Cabs = gold_rows(a, w)
    check_rows(gemm_rows(torch, out, a), C, Cabs)
