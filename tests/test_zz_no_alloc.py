"""bd_w4a6_gemm_noalloc -- the entry point whose stream-K scratch is a static device array in
the library instead of a caller workspace. Collected last (file name) so it runs after every
other GPU test has used the library; it must also pass when run alone. Each case compares two
no-alloc calls in a row with bd_w4a6_gemm on a caller workspace: the results must be the same
bytes (one schedule, one summation order)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _operands(M, N, K, seed):
    import bitdance_b200 as bd
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    a = bd.pack_activations(
        torch.randint(0, 64, (M, K), dtype=torch.uint8, device="cuda", generator=g),
        torch.randint(122, 132, (M, K // 32), dtype=torch.uint8, device="cuda", generator=g))
    w = bd.pack_weights(
        torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g),
        torch.randint(0x30, 0x48, (N, K // 16), dtype=torch.uint8, device="cuda", generator=g),
        0.5)
    return a, w


@pytest.mark.parametrize("M,N,K", [(1, 14336, 4096), (16, 2048, 1024), (5, 1152, 2048),
                                   (32, 4096, 512), (1024, 14336, 512)])
def test_noalloc_matches_the_workspace_entry_point(M, N, K):
    import bitdance_b200 as bd
    a, w = _operands(M, N, K, seed=M + N + K)
    ref = bd.w4a6_gemm(a, w, workspace=bd.Workspace())
    got = []
    for _ in range(2):                       # two calls in a row share the static scratch
        out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        got.append(bd.w4a6_gemm_noalloc(a, w, out))
    torch.cuda.synchronize()
    assert bd.device_error() == 0
    assert ref.abs().max() > 0
    for g in got:
        assert torch.equal(g, ref)


def test_noalloc_bias_epilogue_and_fp32_output():
    import bitdance_b200 as bd
    M, N, K = 8, 1536, 1024
    a, w = _operands(M, N, K, seed=7)
    bias = torch.linspace(-2, 2, N, device="cuda").to(torch.bfloat16)
    ref = bd.w4a6_gemm(a, w, bias=bias, epilogue="bias_relu", out_dtype=torch.float32,
                       workspace=bd.Workspace())
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    bd.w4a6_gemm_noalloc(a, w, out, bias=bias, epilogue="bias_relu")
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_noalloc_rejects_scratch_larger_than_the_static_array():
    import bitdance_b200 as bd
    from bitdance_b200 import _lib
    # 128 token rows per tile, 56 tiles: stream-K scratch of 148 x 2 x 128 x 256 fp32 > 16 MiB
    M, N, K = 128, 14336, 512
    a, w = _operands(M, N, K, seed=11)
    assert bd.query_workspace(M, N, K, 0) > 16 << 20
    out = torch.zeros((M, N), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(bd.BitdanceError) as e:
        bd.w4a6_gemm_noalloc(a, w, out)
    assert e.value.status == _lib.BD_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert not out.any()                     # nothing was launched
