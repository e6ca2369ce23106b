"""Shape sweep of the W4A6 GEMM (the transcode-isolation config's GEMM sweep): every
combination of M, N, K in {256, 1024, 4096}, plus 8192 along each axis, with the first config's
operand distributions (A ~ N(0,1) -> MXFP6, B ~ N(0, 0.02) -> NVFP4 per-16 + fp32 tensor
scale), library-chosen schedule, checked against the oracle's dequantise-then-matmul gold
(max-abs-rel error <= 1e-2 and the elementwise bf16 bound). Quantised operands are cached per
(rows, K) so each matrix is quantised once."""
import functools
import itertools

import numpy as np
import pytest

import w4a6_oracle as o
from test_gemm_gpu import check, run_gpu

pytestmark = pytest.mark.gpu

SIZES = (256, 1024, 4096)
CASES = list(itertools.product(SIZES, SIZES, SIZES)) + [
    (8192, 256, 256), (256, 8192, 256), (256, 256, 8192), (1024, 1024, 8192)]


@functools.lru_cache(maxsize=None)
def acts(M, K):
    return o.quantize_a_mxfp6(o.gen_normal((M, K), 1.0, 0))


@functools.lru_cache(maxsize=None)
def weights(N, K):
    b_codes, b_sc, s_t = o.quantize_b_nvfp4(o.gen_normal((N, K), 0.02, 1), block=16)
    b_packed = o.pack_nibbles(b_codes)
    e6, e8 = o.transcode_b(b_packed, b_sc, 16)
    return b_packed, b_sc, float(s_t), e6, e8


@pytest.mark.parametrize("M,N,K", CASES)
def test_gemm_shape_sweep(M, N, K):
    a_codes, a_e8 = acts(M, K)
    b_packed, b_sc, s_t, e6, e8 = weights(N, K)
    C = o.gemm_gold(a_codes, a_e8, e6, e8, s_t)
    Cabs = o.gemm_gold(a_codes & 0x1F, a_e8, e6 & 0x1F, e8, abs(s_t))
    check(run_gpu(a_codes, a_e8, b_packed, b_sc, s_t), C, Cabs)
