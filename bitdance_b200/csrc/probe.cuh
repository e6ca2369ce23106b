// probe.cuh -- issue-rate probe of the block-scaled tensor-core MMA the W4A6 GEMM is built on
// (tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale, M = 128, K = 32 per instruction):
// the FP6 (= FP8-rate) tensor peak the GEMM's roofline is measured against.
//
// One CTA per SM; one thread issues `n_mma` MMAs back to back into one fp32 accumulator
// (the shape of a GEMM's K loop), operands resident on chip: B (n_cols rows x 128 B of E4M3,
// 128B-swizzled, K-major) in shared memory; A (128 rows x 128 B of E2M3 codes) in shared
// memory (SS form) or tensor memory (TS form, what the GEMM uses); E8M0 scale factors 1.0 in
// tensor memory. The operands are pseudo-random codes (a hash of the byte index): all-zero
// operands run the same cycles per MMA but draw less power, so the clock stays higher than a
// GEMM on real data can hold (3.99 against 3.55 PFLOP/s measured for N = 256, TS form). E4M3
// bytes have bit 6 clear (magnitudes below 2, no NaN); E2M3 codes are any 6-bit value. The host
// times the launch with CUDA events: rate = SMs x n_mma x 2 x 128 x n_cols x 32 / time.
// Plays the part of the reference's MFMA peak probe (kernel/hip/mfma_peak.hip:22-59).
#pragma once
#include "sm100.cuh"

namespace bd {

// B tile + A tile + alignment slack is 49 KB; the launch asks for more dynamic shared memory
// than two CTAs can share, so the grid of one CTA per SM really lands one on every SM (two CTAs
// on one SM would serialise on the tensor-memory allocation while another SM idles).
constexpr int kProbeSmem = 160 * 1024;

__device__ __forceinline__ uint32_t probe_hash(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

__global__ void __launch_bounds__(128, 1)
    mma_peak_kernel(long long n_mma, int n_cols, int a_from_tmem, uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t probe_raw[];
  uint8_t* smem = probe_raw + ((1024u - (smem_u32(probe_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5;

  // B (32 KB of E4M3) and A (16 KB of E2M3 codes, one per byte)
  uint32_t* words = reinterpret_cast<uint32_t*>(smem);
  for (int i = tid; i < 32768 / 4; i += blockDim.x)
    words[i] = probe_hash(static_cast<uint32_t>(i) * 2654435761u + 1u) & 0xBFBFBFBFu;
  for (int i = tid; i < 16384 / 4; i += blockDim.x)
    words[8192 + i] = probe_hash(static_cast<uint32_t>(i) * 40503u + 77u) & 0x3F3F3F3Fu;
  if (tid == 0) {
    mbar_init(smem_u32(&done_bar), 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&tmem_base), 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();  // the operands, written by the generic proxy, are read by the MMA
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = tmem_base;
  // each warp fills its lane quarter: A slot (columns 256..287) with codes, scale factors
  // (columns 288..299: 4 token columns, 8 weight columns) E8M0 127 = 1.0 in every byte
  {
    const uint32_t lane_base = tb + (static_cast<uint32_t>(warp * 32) << 16);
    uint32_t z[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
      z[i] = probe_hash(static_cast<uint32_t>(tid * 32 + i) + 999u) & 0x3F3F3F3Fu;
    tmem_st_x32(lane_base + 256, z);
    const uint32_t one = 0x7F7F7F7Fu;
    tmem_st_x4(lane_base + 288, one, one, one, one);
    const uint32_t ones[8] = {one, one, one, one, one, one, one, one};
    tmem_st_x8(lane_base + 292, ones);
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
    const uint32_t b_addr = smem_u32(smem);
    const uint32_t a_addr = smem_u32(smem + 32768);
    const uint32_t sfa = tb + 288, sfb = tb + 292;
    for (long long i = 0; i < n_mma; ++i) {
      const uint32_t kk = static_cast<uint32_t>(i & 3);
      const uint32_t idesc = idesc_mxf8f6f4(128, static_cast<uint32_t>(n_cols), kFmtE2M3,
                                            kFmtE4M3, kk, kk);
      const uint32_t acc = i > 0 ? 1u : 0u;
      if (a_from_tmem)
        mma_mxf8f6f4_ts(tb, tb + 256 + kk * 8, sdesc_sw128(b_addr + kk * 32), idesc, sfa, sfb,
                        acc);
      else
        mma_mxf8f6f4_ss(tb, sdesc_sw128(a_addr + kk * 32), sdesc_sw128(b_addr + kk * 32), idesc,
                        sfa, sfb, acc);
    }
    tc_commit(smem_u32(&done_bar));
    mbar_wait(smem_u32(&done_bar), 0, err, kErrWaitMma, nullptr);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tb, 512);
  }
}

// The pair form (tcgen05.mma.cta_group::2, M = 256, N = 256, K = 32, A from tensor memory, the
// MMA of the GEMM's CTA-pair tiles): clusters of two CTAs, each holding 128 rows of A and of B
// and its own scale factors; rank 0 issues. Rate = clusters x n_mma x 2 x 256 x 256 x 32 / time.
__global__ void __launch_bounds__(128, 1) mma_peak_pair_kernel(long long n_mma, uint32_t* err) {
  extern __shared__ __align__(1024) uint8_t probe_raw[];
  uint8_t* smem = probe_raw + ((1024u - (smem_u32(probe_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_base;
  const int tid = threadIdx.x, warp = tid >> 5;
  const uint32_t rank = cluster_ctarank();
  // this CTA's 128 rows of B (16 KB of E4M3)
  uint32_t* words = reinterpret_cast<uint32_t*>(smem);
  for (int i = tid; i < 16384 / 4; i += blockDim.x)
    words[i] =
        probe_hash(static_cast<uint32_t>(i + 4096 * rank) * 2654435761u + 1u) & 0xBFBFBFBFu;
  if (tid == 0) {
    mbar_init(smem_u32(&done_bar), 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc_pair(smem_u32(&tmem_base), 512);
    tmem_relinquish_pair();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = tmem_base;
  {
    // A slot (columns 256..287), token scales (288..291: row m at lane m, column m / 32) and
    // weight scales (292..299: all 256 rows in every lane quarter), E8M0 127 = 1.0
    const uint32_t lane_base = tb + (static_cast<uint32_t>(warp * 32) << 16);
    uint32_t z[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
      z[i] = probe_hash(static_cast<uint32_t>(tid * 32 + i + 4096 * rank) + 999u) & 0x3F3F3F3Fu;
    tmem_st_x32(lane_base + 256, z);
    const uint32_t one = 0x7F7F7F7Fu;
    tmem_st_x4(lane_base + 288, one, one, one, one);
    const uint32_t ones[8] = {one, one, one, one, one, one, one, one};
    tmem_st_x8(lane_base + 292, ones);
    tmem_st_wait();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' operands and barriers are in place
  tc_fence_after();
  if (tid == 0) {
    if (rank == 0) {
      const uint32_t b_addr = smem_u32(smem);
      for (long long i = 0; i < n_mma; ++i) {
        const uint32_t kk = static_cast<uint32_t>(i & 3);
        const uint32_t idesc = idesc_mxf8f6f4(256, 256, kFmtE2M3, kFmtE4M3, kk, kk);
        mma_mxf8f6f4_ts_pair(tb, tb + 256 + kk * 8, sdesc_sw128(b_addr + kk * 32), idesc,
                             tb + 288, tb + 292, i > 0 ? 1u : 0u);
      }
      tc_commit_pair(smem_u32(&done_bar), 3);
    }
    mbar_wait(smem_u32(&done_bar), 0, err, kErrWaitMma, nullptr);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA frees its tensor memory while the pair still works
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tb, 512);
  }
}

}  // namespace bd
