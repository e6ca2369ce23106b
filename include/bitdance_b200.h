/*
 * bitdance_b200.h -- C ABI of the B200 (sm_100a) W4A6 GEMM with on-chip NVFP4 -> MXFP6
 * weight transcode.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (passed as
 * `bd_stream_t`, i.e. a `cudaStream_t` cast to `void*`; NULL = legacy default stream),
 * enqueues work on that stream and returns a status code (BD_OK == 0, negative on error)
 * without synchronising. Arguments are validated before anything is launched. No entry
 * point allocates device memory; the caller owns every buffer.
 *
 * Data formats (all buffers are device memory, row-major unless stated):
 *   NVFP4 weights B, "natural" layout:  codes (N, K/2) u8, element 2j in the low nibble of
 *       byte j (E2M1 nibble = sign<<3 | magnitude index); scales (N, K/16) E4M3 bytes (or
 *       (N, K/32) when scale_block == 32); one fp32 tensor scale.
 *   NVFP4 weights B, "tiled" layout used by the GEMM (bd_pack_b produces it; same byte
 *   count as the natural layout, prepared for the on-chip transcode):
 *       codes  [N/128][K/128][128 rows][64 bytes]: in each 32-bit word (elements 0..7 in
 *              nibbles 0..7) the magnitudes stay in nibble bits 0..2 and the sign of element
 *              i sits at bit 8i+7 (i < 4) or 8(i-4)+3 (i >= 4)
 *       scales [N/128][K/128][128 rows][8 bytes]: per 32-block a 16-bit class word made from
 *              its two E4M3 bytes -- bits 0..5 the magnitude-table row (d*8 + mb) of the
 *              16-block with the smaller exponent, bits 6..8 the other's mantissa bits, bit 9
 *              set when the other is the first 16-block, bits 10..14 E8M0 - 118
 *   NVFP4 weights B, "E4M3 sideband" tiled layout (bd_pack_b_e4m3 produces it; the GEMM reads
 *   it with BD_GEMM_B_E4M3): the natural codes and E4M3 scale bytes, only regrouped into the
 *   tiles above, so buffers filled with constant or random bytes mean what they mean in the
 *   reference's layout (kernel/verify_w4a6.py, kernel/bench_sweep.py).
 *   MXFP6 activations A (bd_pack_a produces both from natural codes and scales):
 *       codes  (M, K) u8: one E2M3 code per byte (bits 0..5; bits 6..7 are ignored), the
 *              byte image the tensor core takes from tensor memory.
 *       scales [K/128][Mp4][4] E8M0 bytes, Mp4 = M rounded up to a multiple of 4.
 *   MXFP6 codes in "natural" form (transcode output, bd_pack_a input): one E2M3 code per
 *       byte in bits [5:0] (sign<<5 | exp<<3 | mantissa); E8M0 = exponent + 127.
 */
#ifndef BITDANCE_B200_H_
#define BITDANCE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* bd_stream_t;

/* ---- status codes ------------------------------------------------------------------- */
#define BD_OK 0
#define BD_ERR_INVALID_ARG (-1)  /* null pointer, bad enum value                          */
#define BD_ERR_SHAPE (-2)        /* dimensions not supported (see each entry point)        */
#define BD_ERR_ALIGNMENT (-3)    /* pointer misaligned for the vector/TMA access it needs  */
#define BD_ERR_ARCH (-4)         /* current device is not sm_100 (B200)                    */
#define BD_ERR_CUDA (-5)         /* a CUDA runtime call failed (launch error, ...)         */
#define BD_ERR_WORKSPACE (-6)    /* workspace missing or smaller than bd_query_workspace() */
#define BD_ERR_DEVICE (-7)       /* a kernel reported an error (bounded wait ran out)      */

/* ---- GEMM options --------------------------------------------------------------------- */
#define BD_OUT_BF16 0
#define BD_OUT_F16 1
#define BD_OUT_F32 2

#define BD_EPI_NONE 0
#define BD_EPI_BIAS 1
#define BD_EPI_BIAS_RELU 2
#define BD_EPI_BIAS_SILU 3
#define BD_EPI_BIAS_GELU 4

/* How split-K partial sums are combined (split_k > 1):
 *   BD_SPLIT_REDUCE: fp32 partials in the caller's workspace, then a reduction kernel
 *                    writes C (epilogue applied once, to the full sum).
 *   BD_SPLIT_PLANES: partial plane z is written to c + z*M*N (out dtype); the caller sums.
 *                    Replaces psg_preshuffle_gemm.py split_reduce="planes" (:296-331).
 *   BD_SPLIT_ATOMIC: every split adds its fp32 partial into c (BD_OUT_F32 only, no
 *                    epilogue, c zeroed by the caller; also at split_k == 1).
 *                    Replaces split_reduce="atomic" (psg:2395-2410).                    */
#define BD_SPLIT_REDUCE 0
#define BD_SPLIT_PLANES 1
#define BD_SPLIT_ATOMIC 2

/* Library version (major*10000 + minor*100 + patch). */
int bd_version(void);

/* Human-readable text of a status code. */
const char* bd_status_string(int status);

/* Bits of the device error word (bd_device_error). */
#define BD_DEVERR_WAIT_MASK 0x1Fu  /* a bounded wait of the GEMM ran out (bits 0..4)     */
#define BD_DEVERR_WAIT_TMA 0x01u   /*   ... a consumer's wait for a TMA stage            */
#define BD_DEVERR_NONFINITE 0x20u  /* a quantiser saw a NaN or an infinity               */
#define BD_DEVERR_RANGE 0x40u      /* a scale had no form in the target format          */

/* Reads (and, if clear != 0, resets) the error word that kernels of this library set on
 * the current device: a bounded wait that ran out, non-finite quantiser input. Synchronises
 * the device. Returns BD_OK and stores the word (0 = no error) in *word. */
int bd_device_error(uint32_t* word, int clear);

/* Diagnostic of the bounded waits (no reference counterpart): one CTA whose first warp waits
 * on an mbarrier that nothing arrives at, with a limit of limit_cycles SM cycles, while a
 * second warp waits on another with the GEMM's default limit (about 2 s). The first wait runs
 * out, sets BD_DEVERR_WAIT_TMA in the device error word and raises the CTA's abort flag; the
 * second leaves through that flag. The kernel ends, the context stays usable, and the host
 * reads the status with bd_device_error. 1000 <= limit_cycles <= 4e9. */
int bd_selftest_bounded_wait(int64_t limit_cycles, bd_stream_t stream);

/* Tensor-core peak probe (the FP6 = FP8-rate roofline of the GEMM): one CTA per SM, each
 * issuing mmas_per_cta block-scaled tcgen05.mma.kind::mxf8f6f4 (M = 128, N = n_cols, K = 32,
 * E2M3 x E4M3 operands, E8M0 scales) back to back into one fp32 accumulator, operands on chip;
 * A from shared memory (a_from_tmem == 0) or tensor memory (1, the GEMM's form); 2: the MMA of
 * CTA pairs (tcgen05 cta_group::2, M = 256 over two CTAs of a cluster, A from tensor memory,
 * n_cols == 256; the GEMM's CTA-pair tiles). The caller times the launch on `stream`:
 * rate = SMs * mmas_per_cta * 2 * 128 * n_cols * 32 / time (the pair form: SMs rounded down to
 * even). 1 <= mmas_per_cta <= 2^21; n_cols a multiple of 16 in [16, 256].
 * Replaces the reference's MFMA issue-rate probe (kernel/hip/mfma_peak.hip:22-59). */
int bd_probe_mma_peak(int64_t mmas_per_cta, int n_cols, int a_from_tmem, bd_stream_t stream);

/* NVFP4 -> MXFP6 transcode, global -> global, natural layouts.
 * nblk32 blocks of 32 elements: codes 16 B per block, scales 2 B per block (scale_block 16,
 * the per-16 pair rule) or 1 B per block (scale_block 32), output 32 E2M3 code bytes and one
 * E8M0 byte per block.
 * Replaces the reference's golden_mxfp6 (kernel/nvfp4_codec.py:66-76) and its device forms
 * _tc_bdata_fp4_to_fp6 / _tc_bscale_e4m3_to_e8m0 (psg_preshuffle_gemm.py:1154-1188,
 * 1283-1329). Alignment: codes and e2m3_out 16 B, scales 2 B when scale_block == 16. */
int bd_transcode_nvfp4_to_mxfp6(const uint8_t* codes, const uint8_t* scales, uint8_t* e2m3_out,
                                uint8_t* e8m0_out, int64_t nblk32, int scale_block,
                                bd_stream_t stream);

/* Natural NVFP4 B -> tiled GEMM layout. N % 128 == 0, K % 128 == 0.
 * Replaces the reference's host-side B pre-pack build_Bpk (kernel/hip/w4a6_tc_gemm_v31.hip:617-642)
 * and the preshuffle B layout (ref_aiter_flydsl/mfma_preshuffle_pipeline.py:168-231). */
int bd_pack_b(const uint8_t* codes, const uint8_t* scales16, uint8_t* codes_tiled,
              uint8_t* scales_tiled, int N, int K, bd_stream_t stream);

/* Natural NVFP4 B -> the E4M3-sideband tiled layout (regrouped only; read with BD_GEMM_B_E4M3).
 * Same arguments and checks as bd_pack_b. The layout the reference-facing operator shim takes. */
int bd_pack_b_e4m3(const uint8_t* codes, const uint8_t* scales16, uint8_t* codes_tiled,
                   uint8_t* scales_tiled, int N, int K, bd_stream_t stream);

/* MXFP4 weight scales (one E8M0 byte per 32-block) -> E4M3 scale bytes for both 16-blocks of
 * each block (2 * nblk32 bytes out, in the same order): E8M0 e becomes the E4M3 byte of the
 * power of two 2^(e-127), for which the per-16 pair rule reproduces the MXFP4 block exactly.
 * Turns an MXFP4 weight (E2M1 codes, E8M0 per-32 scales: the reference's in_dtype="w4a6" arm,
 * psg_preshuffle_gemm.py:411-423, the bit-exact cross-check of kernel/verify_w4a6.py:166-172)
 * into NVFP4 bytes the GEMM takes. Exponents e - 127 outside [-9, 8] have no E4M3 form: those
 * blocks get scale 0 and BD_DEVERR_RANGE is set in the device error word. e4m3_pairs 2-byte
 * aligned. */
int bd_scales_e8m0_to_e4m3_pairs(const uint8_t* e8m0, uint8_t* e4m3_pairs, int64_t nblk32,
                                  bd_stream_t stream);

/* Natural MXFP6 A (one code per byte, (M, K/32) E8M0) -> GEMM operand layout. K % 128 == 0.
 * scales_tiled must hold K/32 * Mp4 bytes; padding rows are written as 127 (2^0). The codes are
 * already in the operand layout: a_packed receives a copy with bits 6..7 cleared, and
 * a_packed == codes is allowed (nothing is copied; only the scales are re-laid out).
 * Replaces the reference's A packing (pack6_block, kernel/verify_w4a6.py:55-59;
 * build_Afrag, kernel/hip/w4a6_tc_gemm_v31.hip:608-615). */
int bd_pack_a(const uint8_t* codes, const uint8_t* e8m0, uint8_t* a_packed,
              uint8_t* scales_tiled, int M, int K, bd_stream_t stream);

/* Input element types of bd_quantize_a_mxfp6 and bd_quantize_b_nvfp4. */
#define BD_IN_F32 0
#define BD_IN_BF16 1

/* Activations x (M, K) row-major, fp32 or bf16 -> MXFP6: E2M3 codes (M, K), one per byte (bits
 * 0..5; this is already the GEMM's `a` operand), and the E8M0 exponent of each 32-element
 * block along K, written to e8m0 (natural (M, K/32) layout) and/or scales_tiled (the GEMM's
 * `a_scales` layout of bd_pack_a, K/32 * Mp4 bytes, padding rows 127); either may be NULL,
 * not both. K % 32 == 0 (K % 128 == 0 when scales_tiled is given); x and codes 16-byte
 * aligned.
 * Rule: the block exponent is the smallest e in [-40, 40] with 7.5 * 2^e >= max|x| (a zero
 * block gets e = 0); each x / 2^e goes to the nearest E2M3 magnitude, ties to the lower; the
 * sign bit is kept only on non-zero codes. Bit-identical to the reference's
 * quantize(x, E8M0, E2M3) (vector_quant_error.py:283-319, via the Direct-MXFP6 path :389).
 * The reference refuses NaN / Inf input (:215-252); here such input sets BD_DEVERR_NONFINITE
 * in the device error word (bd_device_error) and the affected blocks' outputs are undefined. */
int bd_quantize_a_mxfp6(const void* x, int x_dtype, uint8_t* codes, uint8_t* e8m0,
                        uint8_t* scales_tiled, int M, int K, bd_stream_t stream);

/* bd_quantize_a_mxfp6 with launch flags: BD_GEMM_OVERLAP_PREV launches it with programmatic
 * stream serialisation (it may be scheduled while the previous kernel on the stream ends, and
 * waits for it before reading x or writing its outputs). Either way the kernel lets a GEMM
 * launched after it with BD_GEMM_OVERLAP_PREV start early (that GEMM reads the codes only
 * after this kernel completes). No reference counterpart. */
int bd_quantize_a_mxfp6_ex(const void* x, int x_dtype, uint8_t* codes, uint8_t* e8m0,
                           uint8_t* scales_tiled, int M, int K, unsigned flags,
                           bd_stream_t stream);

/* Weights w (N, K) row-major, fp32 or bf16 -> NVFP4 with per-16 E4M3 scales and an fp32
 * per-tensor scale, the natural layouts bd_pack_b takes: codes (N, K/2) E2M1 nibbles (element
 * 2j in the low nibble of byte j), scales16 (N, K/16) E4M3 bytes. tstat is a device buffer of
 * two 32-bit words: on return (stream order) tstat[0] holds the tensor scale s_t as a float and
 * tstat[1] the bits of amax(|w|). K % 16 == 0; w 16-byte aligned, codes 8-byte aligned.
 * Rule: s_t = float32(amax / 2688) (1.0 for an all-zero tensor), v = w / s_t in float32; per
 * 16-block the smallest E4M3FN normal >= amax(|v|)/6 (448 at most, 1.0 for a zero block) and the
 * nearest E2M1 magnitude of v / scale, ties to the lower, sign only on non-zero codes.
 * Bit-identical to the reference's two-level NVFP4 encode (run_method,
 * remote/quant_real_weights.py:273-287; encode_nvfp4, kernel/nvfp4_codec.py:34-63). NaN / Inf
 * input sets BD_DEVERR_NONFINITE (the reference raises) and the outputs are undefined. */
int bd_quantize_b_nvfp4(const void* w, int w_dtype, uint8_t* codes, uint8_t* scales16,
                        uint32_t* tstat, int N, int K, bd_stream_t stream);

/* Bytes of workspace bd_w4a6_gemm needs on the current device for this problem.
 * split_k == 0 (stream-K, the default schedule): per-CTA fp32 partial slots plus one arrival
 * counter per output tile. The workspace must be ZEROED before its first use with a given
 * (M, N, K); every call leaves it ready for the next call of the same shape (its counters back
 * at zero). Zero it again before reusing it for another shape (the layout of slots and
 * counters depends on the shape). Calls that run concurrently on the GPU must not share one
 * workspace.
 * split_k > 1 with BD_SPLIT_REDUCE: split_k fp32 planes of M x N. Otherwise 0. */
size_t bd_query_workspace(int M, int N, int K, int split_k, int split_mode);

/* C[M,N] = (A . B^T) * b_tensor_scale (+ bias[N], activation), fp32 accumulation.
 * A: MXFP6 (bd_pack_a layout); B: NVFP4 (bd_pack_b tiled layout), transcoded on chip to MXFP6
 * per the reference contract and fed to block-scaled tcgen05 MMAs.
 * Shapes: M >= 1, N % 128 == 0, K % 128 == 0, (K/128) % split_k == 0 when split_k > 0.
 * split_k == 0: persistent stream-K schedule over (tile, 128-wide K chunk) units, tiles split
 * between CTAs finished in-kernel in a fixed order (needs the workspace, see above).
 * split_k >= 1: each tile's K range cut into split_k pieces; split_mode says how they combine.
 * bias: N bf16 values (used when epilogue != BD_EPI_NONE). With split_mode PLANES, c holds
 * split_k planes; with ATOMIC, out_dtype must be BD_OUT_F32 and epilogue BD_EPI_NONE.
 * Replaces compile_preshuffle_gemm_a8(in_dtype="w4a6_tc") + launch_fn
 * (psg_preshuffle_gemm.py:251-277, 3211-3253) and the HIP kernel `kern`
 * (kernel/hip/w4a6_tc_gemm_v31.hip:152-604). */
int bd_w4a6_gemm(void* c, const uint8_t* a, const uint8_t* a_scales, const uint8_t* b,
                 const uint8_t* b_scales, float b_tensor_scale, const void* bias, int M, int N,
                 int K, int split_k, int split_mode, int out_dtype, int epilogue,
                 void* workspace, size_t workspace_bytes, bd_stream_t stream);

/* Launch flags of bd_w4a6_gemm_ex. */
#define BD_GEMM_OVERLAP_PREV 1u   /* may start while the previous kernel on the stream ends */
#define BD_GEMM_WEIGHTS_STATIC 2u /* b / b_scales are not written by that previous kernel */
#define BD_GEMM_B_E4M3 4u         /* b / b_scales in the E4M3-sideband layout (bd_pack_b_e4m3) */
#define BD_GEMM_SINGLE_CTA 8u     /* no CTA-pair tiles (one CTA per 128-token tile throughout) */

/* bd_w4a6_gemm with launch flags (same arguments, same results). BD_GEMM_B_E4M3: b and b_scales
 * are in the E4M3-sideband layout (bd_pack_b_e4m3) instead of bd_pack_b's; same results for the
 * same natural weights (the transcode then decodes the scale bytes on chip).
 * BD_GEMM_OVERLAP_PREV launches with programmatic stream serialisation: the kernel's CTAs may
 * be scheduled as the previous kernel's CTAs retire (the previous kernel must allow it:
 * bd_w4a6_gemm kernels do, other kernels start it only when they end). The kernel waits for
 * the previous kernel to complete before it reads a, a_scales or bias and before it touches
 * c or the workspace. With BD_GEMM_WEIGHTS_STATIC as well, it starts streaming b and
 * b_scales before that wait, so the caller guarantees that the previous kernel does not
 * write them (weights that stay resident across decode steps). No reference counterpart: the
 * reference launches each GEMM on its own (kernel/bench_sweep.py:87-161).
 * Where whole tiles of 128 tokens fill the machine twice over and N % 256 == 0, tiles of 256
 * tokens x 256 weight rows are computed by clusters of two CTAs sharing each MMA (each CTA
 * transcodes half of every weight chunk); BD_GEMM_SINGLE_CTA keeps one CTA per 128-token tile
 * (same results, bit for bit). */
int bd_w4a6_gemm_ex(void* c, const uint8_t* a, const uint8_t* a_scales, const uint8_t* b,
                    const uint8_t* b_scales, float b_tensor_scale, const void* bias, int M, int N,
                    int K, int split_k, int split_mode, int out_dtype, int epilogue,
                    void* workspace, size_t workspace_bytes, unsigned flags, bd_stream_t stream);

/* bd_w4a6_gemm with split_k = 0 (the default schedule) that allocates nothing and takes no
 * workspace: the stream-K partial slots and tile counters live in a static 16 MiB device array
 * inside the library. For callers that cannot allocate device memory at the call: hosts
 * binding the C ABI without a device allocator of their own, and serving loops whose memory
 * pool is sized up front, where an allocation could synchronise the device or fragment it.
 * Limit: problems whose stream-K scratch (bd_query_workspace(M, N, K, 0, 0)) exceeds 16 MiB
 * return BD_ERR_WORKSPACE (on a 148-SM B200 every problem with M <= 32 fits; problems whose
 * tiles fill the machine twice over need no scratch and always run). Every call clears the
 * tile counters with cudaMemsetAsync on `stream` before the kernel. All calls on a device share
 * the one array: calls that overlap in time (other streams, other threads) race and give
 * wrong results. The first call on each device performs one-time set-up (symbol lookup, kernel
 * attributes); make it before any stream capture. Same results as bd_w4a6_gemm. No reference
 * counterpart (the reference allocates its buffers in Python, kernel/bench_sweep.py:59-85). */
int bd_w4a6_gemm_noalloc(void* c, const uint8_t* a, const uint8_t* a_scales, const uint8_t* b,
                         const uint8_t* b_scales, float b_tensor_scale, const void* bias, int M,
                         int N, int K, int out_dtype, int epilogue, bd_stream_t stream);

/* Sum of split_k fp32 partial planes (split_k, M, N) -> C (out dtype), times b_tensor_scale,
 * plus bias/activation. Replaces the torch.sum over planes in kernel/bench_sweep.py:141-142. */
int bd_splitk_reduce(const float* partials, void* c, const void* bias, float b_tensor_scale,
                     int M, int N, int split_k, int out_dtype, int epilogue, bd_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* BITDANCE_B200_H_ */
