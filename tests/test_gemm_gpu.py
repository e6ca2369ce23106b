"""W4A6 GEMM on the GPU against the oracle's dequantise-then-matmul gold (fp64 accumulation):
C = deq(A) . deq(transcode(B))^T * s_t, max-abs-rel error <= 1e-2,
plus an elementwise bound at bf16 resolution that any layout error would break."""
import numpy as np
import pytest

import w4a6_oracle as o

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TOL_REL_LINF = 1e-2


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def random_operands(M, N, K, seed, b_scale_lo=0x28, b_scale_hi=0x50, a_e8_lo=120, a_e8_hi=134):
    rng = np.random.default_rng(seed)
    a_codes = rng.integers(0, 64, (M, K), dtype=np.uint8)
    a_e8 = rng.integers(a_e8_lo, a_e8_hi + 1, (M, K // 32), dtype=np.uint8)
    b_packed = rng.integers(0, 256, (N, K // 2), dtype=np.uint8)
    b_sc = rng.integers(b_scale_lo, b_scale_hi + 1, (N, K // 16), dtype=np.uint8)
    return a_codes, a_e8, b_packed, b_sc


def quantized_operands(M, N, K, a_seed, b_seed, b_kind="normal", b_std=0.02, outliers=False):
    if b_kind == "normal":
        w = o.gen_normal((N, K), b_std, b_seed)
    else:
        w = o.gen_student_t((N, K), b_std, b_seed)
    x = o.gen_outlier_acts((M, K), a_seed) if outliers else o.gen_normal((M, K), 1.0, a_seed)
    a_codes, a_e8 = o.quantize_a_mxfp6(x)
    b_codes, b_sc, s_t = o.quantize_b_nvfp4(w, block=16)
    return a_codes, a_e8, o.pack_nibbles(b_codes), b_sc, float(s_t)


def gold(a_codes, a_e8, b_packed, b_sc, s_t, bias=None):
    e6, e8 = o.transcode_b(b_packed, b_sc, 16)
    C = o.gemm_gold(a_codes, a_e8, e6, e8, s_t, bias)
    Cabs = o.gemm_gold(a_codes & 0x1F, a_e8, e6 & 0x1F, e8, abs(s_t))
    return C, Cabs


def run_gpu(a_codes, a_e8, b_packed, b_sc, s_t, **kw):
    import bitdance_b200 as bd
    acts = bd.pack_activations(dev(a_codes), dev(a_e8))
    w = bd.pack_weights(dev(b_packed), dev(b_sc), s_t)
    C = bd.w4a6_gemm(acts, w, **kw)
    torch.cuda.synchronize()
    assert bd.device_error() == 0
    return C


def check(C_gpu, C, Cabs, out_dtype=torch.bfloat16):
    g = C_gpu.float().cpu().numpy().astype(np.float64)
    assert np.isfinite(g).all()
    assert np.abs(g).max() > 0, "kernel wrote no output"
    assert o.rel_linf(C, g) <= TOL_REL_LINF
    ulp = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11, torch.float32: 2.0 ** -22}[out_dtype]
    bound = ulp * np.abs(C) + 2.0 ** -20 * Cabs + 1e-30
    bad = np.abs(g - C) > bound
    assert not bad.any(), f"{bad.sum()} elements outside bound; first at {np.argwhere(bad)[0]}"


@pytest.mark.parametrize("M", [1, 4, 16, 17, 32, 64, 100, 128, 200, 256, 300])
def test_random_codes_token_tiles(M):
    N, K = 256, 512
    ops = random_operands(M, N, K, seed=M)
    C, Cabs = gold(*ops, 0.37)
    check(run_gpu(*ops, 0.37, split_k=1), C, Cabs)


@pytest.mark.parametrize("K", [128, 256, 384, 1024, 2176])
def test_k_lengths_shorter_and_longer_than_the_pipeline(K):
    M, N = 24, 384
    ops = random_operands(M, N, K, seed=K)
    C, Cabs = gold(*ops, 1.0)
    check(run_gpu(*ops, 1.0, split_k=1), C, Cabs)


def test_full_range_scales_with_subnormals_and_large_exponent_gaps():
    M, N, K = 48, 256, 1024
    ops = random_operands(M, N, K, seed=9, b_scale_lo=0x01, b_scale_hi=0x7E, a_e8_lo=100,
                          a_e8_hi=150)
    C, Cabs = gold(*ops, 2.0 ** -10)
    check(run_gpu(*ops, 2.0 ** -10, split_k=1), C, Cabs)


@pytest.mark.parametrize("split_k,mode", [(2, "reduce"), (4, "reduce"), (8, "reduce"),
                                          (4, "planes"), (4, "atomic"), (1, "atomic")])
def test_split_k_modes(split_k, mode):
    M, N, K = 20, 512, 1024
    ops = random_operands(M, N, K, seed=11 + split_k)
    C, Cabs = gold(*ops, 0.5)
    out_dtype = torch.float32 if mode == "atomic" else torch.bfloat16
    got = run_gpu(*ops, 0.5, split_k=split_k, split_mode=mode, out_dtype=out_dtype)
    if mode == "planes":
        assert got.shape == (split_k, M, N)
        got = got.float().sum(0)
        C_ok = o.rel_linf(C, got.cpu().numpy()) <= TOL_REL_LINF
        assert C_ok
        return
    check(got, C, Cabs, out_dtype)


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_output_dtypes(out_dtype):
    M, N, K = 40, 256, 512
    ops = random_operands(M, N, K, seed=21, b_scale_lo=0x20, b_scale_hi=0x38)
    C, Cabs = gold(*ops, 0.01)
    check(run_gpu(*ops, 0.01, split_k=1, out_dtype=out_dtype), C, Cabs, out_dtype)


@pytest.mark.parametrize("epi", ["bias", "bias_relu", "bias_silu", "bias_gelu"])
@pytest.mark.parametrize("split_k", [1, 4])
def test_epilogues(epi, split_k):
    M, N, K = 33, 256, 1024
    ops = random_operands(M, N, K, seed=31, b_scale_lo=0x18, b_scale_hi=0x30)
    bias = (np.random.default_rng(5).standard_normal(N) * 4).astype(np.float32)
    bias_bf = torch.from_numpy(bias).to(torch.bfloat16)
    b64 = bias_bf.float().numpy().astype(np.float64)
    C, Cabs = gold(*ops, 0.05, b64)
    if epi == "bias_relu":
        C = np.maximum(C, 0)
    elif epi == "bias_silu":
        C = C / (1 + np.exp(-C))
    elif epi == "bias_gelu":
        C = 0.5 * C * (1 + np.tanh(np.sqrt(2 / np.pi) * (C + 0.044715 * C ** 3)))
    got = run_gpu(*ops, 0.05, split_k=split_k, bias=bias_bf.cuda(), epilogue=epi)
    g = got.float().cpu().numpy()
    assert o.rel_linf(C, g) <= TOL_REL_LINF
    assert np.abs(g - C).max() <= 2.0 ** -7 * np.abs(C).max() + 1e-3


def test_config1_quantized_normal():
    """M=128, N=4096, K=4096; A ~ N(0,1) seed 0 -> MXFP6, B ~ N(0,0.02)
    seed 1 -> NVFP4 per-16 + fp32 tensor scale."""
    a_codes, a_e8, b_packed, b_sc, s_t = quantized_operands(128, 4096, 4096, 0, 1)
    C, Cabs = gold(a_codes, a_e8, b_packed, b_sc, s_t)
    check(run_gpu(a_codes, a_e8, b_packed, b_sc, s_t), C, Cabs)


@pytest.mark.parametrize("M", [1, 4, 16, 32, 64])
def test_config2_decode_shapes(M):
    """BASELINE config 2 distributions (Student-t weights, outlier activations), N reduced to
    2048 for the oracle; K = 4096 as in the config; library-chosen split-K."""
    a_codes, a_e8, b_packed, b_sc, s_t = quantized_operands(M, 2048, 4096, 3 + M, 2,
                                                            b_kind="t", outliers=True)
    C, Cabs = gold(a_codes, a_e8, b_packed, b_sc, s_t)
    check(run_gpu(a_codes, a_e8, b_packed, b_sc, s_t, split_k=0), C, Cabs)


def test_verify_w4a6_constant_operands():
    """kernel/verify_w4a6.py: constant-along-K operands give C = K * a * b * b_scale
    (:122-193); byte-uniform A 0x55 decodes to +3.25 in every 6-bit slot (:81-97)."""
    import bitdance_b200 as bd
    M, N, K = 128, 256, 2048
    a = torch.full((M, K), 0x55, dtype=torch.uint8, device="cuda")   # already operand layout
    a_sc = torch.full(((K // 32) * M,), 127, dtype=torch.uint8, device="cuda")
    acts = bd.PackedActivations(a, a_sc, M, K)
    bc = o.E2M1_POS.tolist().index(2.0)
    for b_scale, byte in ((1.0, 0x38), (1.5, 0x3C), (0.5, 0x30)):
        w = bd.pack_weights(torch.full((N, K // 2), (bc << 4) | bc, dtype=torch.uint8, device="cuda"),
                            torch.full((N, K // 16), byte, dtype=torch.uint8, device="cuda"), 1.0)
        C = bd.w4a6_gemm(acts, w, split_k=1).float().cpu().numpy()
        # the transcode folds the scale mantissa: 1.5 * 2 = 3 -> E2M3 1.5 * 2^1 exactly
        expected = K * 3.25 * 2.0 * b_scale
        assert np.all(np.abs(C - expected) <= 1e-3 * abs(expected)), (b_scale, C[:2, :3])


def test_rejects_unsupported_shapes_and_small_workspace():
    import bitdance_b200 as bd
    from bitdance_b200 import BitdanceError, _lib
    ops = random_operands(16, 256, 512, seed=1)
    acts = bd.pack_activations(dev(ops[0]), dev(ops[1]))
    w = bd.pack_weights(dev(ops[2]), dev(ops[3]), 1.0)
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(BitdanceError) as e:
        bd.w4a6_gemm(acts, w, split_k=4, split_mode="reduce", workspace=ws)
    assert e.value.status == _lib.BD_ERR_WORKSPACE
    with pytest.raises(BitdanceError) as e:
        bd.w4a6_gemm(acts, w, split_k=0, workspace=ws)
    assert e.value.status == _lib.BD_ERR_WORKSPACE
    with pytest.raises(BitdanceError) as e:
        bd.w4a6_gemm(acts, w, split_k=3)
    assert e.value.status == _lib.BD_ERR_SHAPE


@pytest.mark.parametrize("M,N,K", [(16, 2048, 4096), (64, 256, 4096), (1, 128, 128),
                                   (300, 384, 1024), (16, 14336, 1024), (5, 1024, 8192),
                                   (129, 640, 2048)])
def test_streamk_schedule(M, N, K):
    """Default schedule: tiles split between CTAs (up to 32 contributors per tile), fixed up
    in-kernel; repeated calls reuse the workspace and give bit-identical results."""
    import bitdance_b200 as bd
    ops = random_operands(M, N, K, seed=M + N + K)
    C, Cabs = gold(*ops, 0.75)
    acts = bd.pack_activations(dev(ops[0]), dev(ops[1]))
    w = bd.pack_weights(dev(ops[2]), dev(ops[3]), 0.75)
    ws = bd.Workspace()
    first = bd.w4a6_gemm(acts, w, workspace=ws)
    second = bd.w4a6_gemm(acts, w, workspace=ws)
    torch.cuda.synchronize()
    assert bd.device_error() == 0
    check(first, C, Cabs)
    assert torch.equal(first, second)
    # the arrival counters (the tail of the workspace) are back at zero after every call
    nbytes = bd.query_workspace(M, N, K, 0)
    bn = 16 if M <= 16 else 32 if M <= 32 else 64 if M <= 64 else 128 if M <= 128 else 256
    tiles = (N // 128) * ((M + bn - 1) // bn)
    counter_bytes = (tiles * 4 + 255) // 256 * 256
    assert int(ws.buf[nbytes - counter_bytes:nbytes].count_nonzero()) == 0


def test_streamk_epilogues_and_dtypes():
    M, N, K = 24, 512, 2048
    ops = random_operands(M, N, K, seed=77, b_scale_lo=0x18, b_scale_hi=0x30)
    bias = (np.random.default_rng(6).standard_normal(N) * 4).astype(np.float32)
    bias_bf = torch.from_numpy(bias).to(torch.bfloat16)
    C, Cabs = gold(*ops, 0.05, bias_bf.float().numpy().astype(np.float64))
    C = C * 0.5 * (1 + np.tanh(0.5 * C))   # SiLU without overflow
    got = run_gpu(*ops, 0.05, bias=bias_bf.cuda(), epilogue="bias_silu", out_dtype=torch.float16)
    g = got.float().cpu().numpy()
    assert o.rel_linf(C, g) <= TOL_REL_LINF


def test_workspace_reused_across_shapes():
    """One Workspace serving several problem shapes in turn (it re-zeroes on a shape change)."""
    import bitdance_b200 as bd
    ws = bd.Workspace()
    for i, (M, N, K) in enumerate([(128, 4096, 1024), (1, 2048, 4096), (16, 2048, 4096),
                                   (128, 4096, 1024), (16, 2048, 4096)]):
        ops = random_operands(M, N, K, seed=100 + i)
        C, Cabs = gold(*ops, 1.0)
        acts = bd.pack_activations(dev(ops[0]), dev(ops[1]))
        w = bd.pack_weights(dev(ops[2]), dev(ops[3]), 1.0)
        check(bd.w4a6_gemm(acts, w, workspace=ws), C, Cabs)


@pytest.mark.parametrize("M", [1, 16, 64, 200])
def test_overlapped_launch_chain(M):
    """GEMMs launched with programmatic serialisation (bd_w4a6_gemm_ex flags): a chain where
    every GEMM shares C and the stream-K workspace with the one before it, and where each
    activation matrix is written by the kernel right before its GEMM, gives the same bytes as
    the same chain launched one after another, and each matches the gold."""
    import bitdance_b200 as bd
    N, K = 1024, 2048
    n_chain = 6
    ops_list = [random_operands(M, N, K, seed=100 * M + i) for i in range(n_chain)]
    ws = [bd.pack_weights(dev(op[2]), dev(op[3]), 0.5) for op in ops_list]
    a_nat = [(dev(op[0]), dev(op[1])) for op in ops_list]
    for overlap in (False, True):
        wsp = bd.ops.Workspace()
        out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        got = []
        for i in range(n_chain):
            acts = bd.pack_activations(*a_nat[i])          # written by the previous kernel
            bd.w4a6_gemm(acts, ws[i], out=out, workspace=wsp, overlap_prev=overlap,
                         weights_static=overlap)
            bd.w4a6_gemm(acts, ws[(i + 1) % n_chain], out=out, workspace=wsp,
                         overlap_prev=overlap, weights_static=overlap)
            got.append(out.clone())
        torch.cuda.synchronize()
        assert bd.device_error() == 0
        if not overlap:
            ref = got
        else:
            for i in range(n_chain):
                assert torch.equal(got[i], ref[i]), i
    for i in (0, n_chain - 1):
        a_codes, a_e8 = ops_list[i][0], ops_list[i][1]
        b_packed, b_sc = ops_list[(i + 1) % n_chain][2], ops_list[(i + 1) % n_chain][3]
        C, Cabs = gold(a_codes, a_e8, b_packed, b_sc, 0.5)
        check(ref[i], C, Cabs)



@pytest.mark.parametrize("split_k", [0, 2])
def test_repeated_calls_are_bitwise_identical(split_k):
    """Stream-K (split_k=0) and split-K results are the same bytes on every call, also with a
    freshly zeroed workspace each time (stale partials from an earlier call cannot mask a
    partial that is read too early). Decode shape with three-way split tiles."""
    import bitdance_b200 as bd
    M, N, K = 16, 14336, 4096
    a_codes, a_e8, b_packed, b_sc = random_operands(M, N, K, seed=77)
    acts = bd.pack_activations(dev(a_codes), dev(a_e8))
    w = bd.pack_weights(dev(b_packed), dev(b_sc), 0.5)
    ref = bd.w4a6_gemm(acts, w, split_k=split_k, workspace=bd.Workspace()).clone()
    ws = bd.Workspace()
    for i in range(60):
        got = bd.w4a6_gemm(acts, w, split_k=split_k,
                           workspace=bd.Workspace() if i % 2 else ws)
        assert torch.equal(got, ref), f"call {i} differs"
    torch.cuda.synchronize()
    assert bd.device_error() == 0


@pytest.mark.parametrize("M,N,K", [(128, 14336, 4096), (1024, 4096, 4096), (16, 14336, 8192),
                                   (32, 14336, 8192)])
def test_streamk_long_segments_full_token_tile(M, N, K):
    """Stream-K with 12..27 K chunks per CTA (128-row token tiles) and 24 per CTA (16- and
    32-row decode tiles): most CTAs run the tail of one tile, store its partial, then start
    the next tile while the rings are full.
    Every call is checked against the oracle (a weight stage released before its reads were
    performed showed up here as rows converted from a later chunk, on some calls only)."""
    import bitdance_b200 as bd
    a_codes, a_e8, b_packed, b_sc = random_operands(M, N, K, seed=M + 5)
    C, Cabs = gold(a_codes, a_e8, b_packed, b_sc, 1.0)
    acts = bd.pack_activations(dev(a_codes), dev(a_e8))
    w = bd.pack_weights(dev(b_packed), dev(b_sc), 1.0)
    ws = bd.Workspace()
    first = None
    for i in range(4):
        got = bd.w4a6_gemm(acts, w, out_dtype=torch.float32, workspace=ws)
        check(got, C, Cabs, torch.float32)
        if first is None:
            first = got.clone()
        assert torch.equal(got, first), f"call {i} differs"
    assert bd.device_error() == 0


@pytest.mark.parametrize("M,split_k", [(5, 0), (24, 0), (200, 1), (512, 1), (300, 0)])
def test_pack_activations_in_place_gives_the_same_gemm(M, split_k):
    """pack_activations(..., inplace=True) uses the natural codes as the operand (only the scales
    are re-laid out) and gives the same result as the copying form, also with bits 6..7 of the
    code bytes set (the GEMM ignores them): 16- and 32-row decode tiles (M = 5, 24), CTA-pair
    tiles (M = 200, 512 with whole tiles) and 128-row tiles (M = 300, stream-K)."""
    import bitdance_b200 as bd
    N, K = 512, 1024
    a_codes, a_e8, b_packed, b_sc = random_operands(M, N, K, seed=41 + M)
    junk = (np.random.default_rng(M).integers(0, 4, a_codes.shape) << 6).astype(np.uint8)
    w = bd.pack_weights(dev(b_packed), dev(b_sc), 1.0)
    ref = bd.w4a6_gemm(bd.pack_activations(dev(a_codes), dev(a_e8)), w, split_k=split_k)
    codes = dev(a_codes | junk)
    packed = bd.pack_activations(codes, dev(a_e8), inplace=True)
    assert packed.codes.data_ptr() == codes.data_ptr()
    got = bd.w4a6_gemm(packed, w, split_k=split_k)
    torch.cuda.synchronize()
    assert bd.device_error() == 0
    assert torch.equal(got, ref)
    C, Cabs = gold(a_codes, a_e8, b_packed, b_sc, 1.0)
    check(got.float(), C, Cabs, torch.bfloat16)


@pytest.mark.parametrize("M,N,K,split_k", [(16, 2048, 4096, 0), (1, 14336, 1024, 0),
                                           (128, 1024, 2048, 1), (300, 768, 1024, 2)])
def test_both_weight_layouts_give_the_same_bytes(M, N, K, split_k):
    """bd_pack_b's transcode-ready layout (moved sign bits, class words) and the E4M3 sideband
    (bd_pack_b_e4m3, read with BD_GEMM_B_E4M3) produce the same B tile on chip, so the GEMM
    results are identical; full-range scale bytes (subnormal and zero scales, large gaps)."""
    import bitdance_b200 as bd
    ops = random_operands(M, N, K, seed=M + N + K + split_k, b_scale_lo=0x00, b_scale_hi=0x7E)
    acts = bd.pack_activations(dev(ops[0]), dev(ops[1]))
    out = []
    for sideband in ("class", "e4m3"):
        w = bd.pack_weights(dev(ops[2]), dev(ops[3]), 0.5, sideband=sideband)
        out.append(bd.w4a6_gemm(acts, w, split_k=split_k, out_dtype=torch.float32).clone())
    torch.cuda.synchronize()
    assert bd.device_error() == 0
    assert torch.equal(out[0], out[1])
    C, Cabs = gold(*ops, 0.5)
    check(out[0], C, Cabs, torch.float32)


@pytest.mark.parametrize("M,out_dtype,epi", [(200, torch.float16, "bias_gelu"),
                                             (300, torch.bfloat16, "bias_relu"),
                                             (129, torch.float16, "none")])
def test_token_tiles_of_128_rows_store_paths(M, out_dtype, epi):
    """128-row token tiles write C with TMA stores from shared memory: 16-bit outputs with an
    epilogue, rows past M left untouched (C is a view into a larger buffer with guard rows),
    and the same values through the per-thread store path when C is not 16-byte aligned."""
    import bitdance_b200 as bd
    N, K = 512, 512
    ops = random_operands(M, N, K, seed=M + 5, b_scale_lo=0x18, b_scale_hi=0x30)
    bias = (np.random.default_rng(M).standard_normal(N) * 2).astype(np.float32)
    bias_bf = torch.from_numpy(bias).to(torch.bfloat16)
    C, Cabs = gold(*ops, 0.05, bias_bf.float().numpy().astype(np.float64) if epi != "none" else None)
    if epi == "bias_relu":
        C = np.maximum(C, 0)
    elif epi == "bias_gelu":
        C = 0.5 * C * (1 + np.tanh(0.7978845608028654 * (C + 0.044715 * C ** 3)))
    acts = bd.pack_activations(dev(ops[0]), dev(ops[1]))
    w = bd.pack_weights(dev(ops[2]), dev(ops[3]), 0.05)
    kw = dict(out_dtype=out_dtype, split_k=1, epilogue=epi,
              bias=bias_bf.cuda() if epi != "none" else None)
    big = torch.full((M + 8, N), float("nan"), dtype=out_dtype, device="cuda")
    got = bd.w4a6_gemm(acts, w, out=big[:M], **kw)
    # the same GEMM into a C that starts 2 bytes past a 16-byte boundary
    flat = torch.full((M * N + 8,), float("nan"), dtype=out_dtype, device="cuda")
    odd = bd.w4a6_gemm(acts, w, out=flat[1:1 + M * N].view(M, N), **kw)
    torch.cuda.synchronize()
    assert bd.device_error() == 0
    assert bool(torch.isnan(big[M:]).all()), "rows past M were written"
    assert bool(torch.isnan(flat[0])) and bool(torch.isnan(flat[1 + M * N:]).all())
    g = got.float().cpu().numpy().astype(np.float64)
    assert o.rel_linf(C, g) <= TOL_REL_LINF
    assert torch.equal(got, odd)


@pytest.mark.parametrize("M,N,K,out_dtype,epi,sideband", [
    (2400, 4096, 512, torch.bfloat16, "none", "class"),      # last pair tile: rank 1 has no rows
    (2440, 4096, 256, torch.float16, "bias_gelu", "class"),  # rank 1 holds 8 rows of the last tile
    (2560, 4096, 128, torch.float32, "bias", "class"),       # one chunk per tile; fp32 C (no TMA store)
    (2432, 4096, 384, torch.bfloat16, "bias_relu", "e4m3"),  # E4M3 sideband
])
def test_cta_pair_tiles(M, N, K, out_dtype, epi, sideband):
    """Whole tiles that fill the machine twice over run as 256-token tiles on CTA pairs (the
    pair MMA, each CTA transcoding half of every weight chunk): against the oracle, and the same
    bits as the single-CTA schedule (BD_GEMM_SINGLE_CTA)."""
    import bitdance_b200 as bd
    ops = random_operands(M, N, K, seed=M + K, b_scale_lo=0x18, b_scale_hi=0x30)
    bias = (np.random.default_rng(K).standard_normal(N) * 2).astype(np.float32)
    bias_bf = torch.from_numpy(bias).to(torch.bfloat16)
    C, Cabs = gold(*ops, 0.05, bias_bf.float().numpy().astype(np.float64) if epi != "none" else None)
    if epi == "bias_relu":
        C = np.maximum(C, 0)
    elif epi == "bias_gelu":
        C = 0.5 * C * (1 + np.tanh(0.7978845608028654 * (C + 0.044715 * C ** 3)))
    acts = bd.pack_activations(dev(ops[0]), dev(ops[1]))
    w = bd.pack_weights(dev(ops[2]), dev(ops[3]), 0.05, sideband=sideband)
    kw = dict(out_dtype=out_dtype, epilogue=epi, bias=bias_bf.cuda() if epi != "none" else None)
    pair = bd.w4a6_gemm(acts, w, **kw)
    single = bd.w4a6_gemm(acts, w, single_cta=True, **kw)
    torch.cuda.synchronize()
    assert bd.device_error() == 0
    g = pair.float().cpu().numpy().astype(np.float64)
    assert np.isfinite(g).all()
    assert o.rel_linf(C, g) <= TOL_REL_LINF
    assert torch.equal(pair, single)
