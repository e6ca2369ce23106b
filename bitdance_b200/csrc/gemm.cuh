// gemm.cuh -- fused W4A6 GEMM for sm_100a: C = A_mxfp6 . transcode(B_nvfp4)^T.
//
// One CTA computes a 128 (weight rows, N) x BN (tokens, M) tile of C^T in tensor memory:
// the weights are the MMA's M operand and the tokens its N operand, so a decode batch of a
// few tokens still fills 128-row MMAs. Per 128-wide K chunk ("stage"):
//
//   warp 0      producer   bulk copies of the packed NVFP4 codes (8 KB) and E4M3 scales
//                          (1 KB) from the tiled B layout, TMA tensor loads of the token
//                          tile (128B-swizzled) and of its E8M0 scales; one mbarrier.
//   warps 2..9  transcode  NVFP4 -> MXFP6 of the 128x128 weight chunk straight into the
//                          128B-swizzled operand buffer (values as E4M3 bytes), the weight
//                          E8M0 scales and the token scales into tcgen05.cp layout.
//   warp 1      MMA        tcgen05.cp of both scale blocks to TMEM, 4 block-scaled
//                          tcgen05.mma (kind::mxf8f6f4, K = 32 each), commit frees the stage.
//   warps 2..9  epilogue   TMEM -> registers -> (x tensor scale, bias, activation) -> C.
//
// Split-K: blockIdx.z covers K/split_k; partial results go to the workspace, to planes of C
// or are added atomically, as the host asks.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include "sm100.cuh"
#include "transcode.cuh"

namespace bd {

enum : int {
  kOutC = 0,       // final values into C (out dtype)
  kOutPartial = 1, // raw fp32 partials into workspace plane z
  kOutPlane = 2,   // scaled partials into plane z of C (out dtype)
  kOutAtomic = 3,  // scaled partials added into fp32 C
};

struct GemmParams {
  const uint8_t* wcodes;   // [N/128][K/128][128][64]
  const uint8_t* wscales;  // [N/128][K/128][128][8]
  void* out;               // C, or workspace for kOutPartial
  const __nv_bfloat16* bias;
  float tensor_scale;
  int M, N, K;
  int ktiles;              // 128-wide K chunks per split
  int out_mode, out_dtype, epilogue;
  uint32_t* err;
};

constexpr int cround(int x, int a) { return (x + a - 1) / a * a; }
constexpr int cpow2(int x) {
  int p = 32;
  while (p < x) p *= 2;
  return p;
}

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN >= 256 ? 3 : (BN >= 128 ? 5 : (BN >= 64 ? 6 : 7));
  static constexpr int kW8 = 128 * 128;
  static constexpr int kA = BN * 128;
  static constexpr int kWCode = 128 * 64;
  static constexpr int kWScale = 128 * 8;
  static constexpr int kAScale = BN * 4;
  static constexpr int kSfA = BN > 128 ? 1024 : 512;
  static constexpr int oW8 = 0;
  static constexpr int oA = oW8 + kW8;
  static constexpr int oWCode = oA + kA;
  static constexpr int oWScale = oWCode + kWCode;
  static constexpr int oAScale = oWScale + kWScale;
  static constexpr int oSfW = cround(oAScale + kAScale, 128);
  static constexpr int oSfA = oSfW + 512;
  static constexpr int kStageBytes = cround(oSfA + kSfA, 1024);
  static constexpr int kTxBytes = kWCode + kWScale + kA + kAScale;
  static constexpr int kSfCols = 4 + (BN > 128 ? 8 : 4);
  static constexpr int kSfCol0 = BN < 32 ? 32 : BN;
  static constexpr int kTmemCols = cpow2(kSfCol0 + kStages * kSfCols);
  // control block after the stages
  static constexpr int oCtl = kStages * kStageBytes;
  static constexpr int kCtlBytes = 1024;
  static constexpr int kSmemBytes = oCtl + kCtlBytes + 1024;  // + alignment slack
  static constexpr int kThreads = 320;
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kTmemCols <= 512, "tensor memory budget");
};

struct GemmCtl {
  uint64_t full[8], ready[8], empty[8], accum;
  uint32_t tmem_base;
  uint32_t abort_flag;
  TranscodeTables tab;
};

__device__ __forceinline__ float apply_epilogue(float v, int epi, const __nv_bfloat16* bias,
                                                int n) {
  if (epi != 0) v += __bfloat162float(bias[n]);
  if (epi == 2) v = fmaxf(v, 0.0f);
  else if (epi == 3) v = v / (1.0f + expf(-v));
  else if (epi == 4) {
    const float y = 0.7978845608028654f * (v + 0.044715f * v * v * v);
    v = 0.5f * v * (1.0f + tanhf(y));
  }
  return v;
}

__device__ __forceinline__ void store_out(void* out, int64_t idx, float v, int dtype) {
  if (dtype == 0) reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  else if (dtype == 1) reinterpret_cast<__half*>(out)[idx] = __float2half_rn(v);
  else reinterpret_cast<float*>(out)[idx] = v;
}

template <int BN>
__global__ void __launch_bounds__(320, 1)
    w4a6_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_as, const GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  GemmCtl& ctl = *reinterpret_cast<GemmCtl*>(smem + Cfg::oCtl);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tile = blockIdx.x, m0 = blockIdx.y * BN, split = blockIdx.z;
  const int n0 = n_tile * 128;
  const int nkt_total = p.K / 128;
  const int kt0 = split * p.ktiles;
  const int nk = p.ktiles;
  volatile uint32_t* abort_flag = &ctl.abort_flag;

  if (tid == 0) {
    ctl.abort_flag = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&ctl.full[s]), 1);
      mbar_init(smem_u32(&ctl.ready[s]), 8);
      mbar_init(smem_u32(&ctl.empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl.accum), 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_as);
  }
  load_tables<true>(ctl.tab, tid, Cfg::kThreads);
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl.tmem_base), Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = ctl.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      const uint8_t* wc = p.wcodes + (static_cast<int64_t>(n_tile) * nkt_total + kt0) * 8192;
      const uint8_t* ws = p.wscales + (static_cast<int64_t>(n_tile) * nkt_total + kt0) * 1024;
      for (int i = 0; i < nk; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(smem_u32(&ctl.empty[s]), ph ^ 1u, p.err, kErrWaitEmpty, abort_flag)) break;
        uint8_t* st = smem + s * Cfg::kStageBytes;
        const uint32_t fb = smem_u32(&ctl.full[s]);
        mbar_arrive_expect_tx(fb, Cfg::kTxBytes);
        bulk_load(smem_u32(st + Cfg::oWCode), wc + static_cast<int64_t>(i) * 8192, 8192, fb);
        bulk_load(smem_u32(st + Cfg::oWScale), ws + static_cast<int64_t>(i) * 1024, 1024, fb);
        tma_load_2d(smem_u32(st + Cfg::oA), &tm_a, (kt0 + i) * 128, m0, fb);
        tma_load_2d(smem_u32(st + Cfg::oAScale), &tm_as, m0, kt0 + i, fb);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t tD = tbase;
      for (int i = 0; i < nk; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(smem_u32(&ctl.ready[s]), ph, p.err, kErrWaitOperand, abort_flag)) break;
        tc_fence_after();
        uint8_t* st = smem + s * Cfg::kStageBytes;
        const uint32_t tSfW = tbase + Cfg::kSfCol0 + s * Cfg::kSfCols;
        const uint32_t tSfA = tSfW + 4;
        tmem_cp_32x128b_x4(tSfW, sdesc_plain(smem_u32(st + Cfg::oSfW), 0, 128));
        tmem_cp_32x128b_x4(tSfA, sdesc_plain(smem_u32(st + Cfg::oSfA), 0, 128));
        if constexpr (BN > 128)
          tmem_cp_32x128b_x4(tSfA + 4, sdesc_plain(smem_u32(st + Cfg::oSfA + 512), 0, 128));
        const uint32_t aw = smem_u32(st + Cfg::oW8), ab = smem_u32(st + Cfg::oA);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t idesc = idesc_mxf8f6f4(128, BN, kFmtE4M3, kFmtE2M3, kk, kk);
          mma_mxf8f6f4_ss(tD, sdesc_sw128(aw + kk * 32), sdesc_sw128(ab + kk * 32), idesc, tSfW,
                          tSfA, (i > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(smem_u32(&ctl.empty[s]));
      }
      tc_commit(smem_u32(&ctl.accum));
    }
  } else {
    // ------------------------------------------------------------------ transcode
    const int t = warp - 2;
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1;
      if (!mbar_wait(smem_u32(&ctl.full[s]), ph, p.err, kErrWaitTma, abort_flag)) break;
      uint8_t* st = smem + s * Cfg::kStageBytes;
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int row = pass * 64 + t * 8 + (lane >> 2);
        const int blk = lane & 3;
        const uint4 q = *reinterpret_cast<const uint4*>(st + Cfg::oWCode + row * 64 + blk * 16);
        const uint32_t sc =
            *reinterpret_cast<const uint16_t*>(st + Cfg::oWScale + row * 8 + blk * 2);
        uint2 T0, T1;
        uint32_t e8;
        scale_pair(ctl.tab, sc & 0xFFu, sc >> 8, T0, T1, e8);
        uint4 o0, o1;
        transcode32<true>(q, T0, T1, o0, o1);
        *reinterpret_cast<uint4*>(st + Cfg::oW8 + sw128_offset(row, blk * 2)) = o0;
        *reinterpret_cast<uint4*>(st + Cfg::oW8 + sw128_offset(row, blk * 2 + 1)) = o1;
        st[Cfg::oSfW + sf_offset(row, blk)] = static_cast<uint8_t>(e8);
      }
      if (t == 0) {
        const uint32_t* raw = reinterpret_cast<const uint32_t*>(st + Cfg::oAScale);
        uint32_t* pat = reinterpret_cast<uint32_t*>(st + Cfg::oSfA);
#pragma unroll
        for (int n = lane; n < BN; n += 32)
          pat[(n >> 7) * 128 + (n & 31) * 4 + ((n >> 5) & 3)] = raw[n];
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.ready[s]));
    }

    // ------------------------------------------------------------------ epilogue
    const bool ok = mbar_wait(smem_u32(&ctl.accum), 0, p.err, kErrWaitAccum, abort_flag);
    tc_fence_after();
    if (ok) {
      const int q = warp & 3;
      const int half = t >> 2;
      const int n = n0 + q * 32 + lane;
      constexpr int kHalf = BN / 2;
      const uint32_t taddr = tbase + (static_cast<uint32_t>(q * 32) << 16);
      for (int c0 = half * kHalf; c0 < (half + 1) * kHalf; c0 += 8) {
        if (m0 + c0 >= p.M) break;  // uniform across the warp
        uint32_t r[8];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
              "=r"(r[6]), "=r"(r[7])
            : "r"(taddr + c0));
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int m = m0 + c0 + j;
          if (m < p.M) {
            const float acc = __uint_as_float(r[j]);
            if (p.out_mode == kOutC) {
              const float v = apply_epilogue(acc * p.tensor_scale, p.epilogue, p.bias, n);
              store_out(p.out, static_cast<int64_t>(m) * p.N + n, v, p.out_dtype);
            } else if (p.out_mode == kOutPartial) {
              reinterpret_cast<float*>(p.out)[(static_cast<int64_t>(split) * p.M + m) * p.N + n] =
                  acc;
            } else if (p.out_mode == kOutPlane) {
              store_out(p.out, (static_cast<int64_t>(split) * p.M + m) * p.N + n,
                        acc * p.tensor_scale, p.out_dtype);
            } else {
              atomicAdd(reinterpret_cast<float*>(p.out) + static_cast<int64_t>(m) * p.N + n,
                        acc * p.tensor_scale);
            }
          }
        }
      }
    }
  }

  // ------------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) mbar_wait(smem_u32(&ctl.accum), 0, p.err, kErrWaitAccum, nullptr);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tbase, Cfg::kTmemCols);
  }
}

// Sum of fp32 partial planes -> C with scale, bias and activation. Vectorised by 4 along N.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, void* __restrict__ out,
                                     const __nv_bfloat16* __restrict__ bias, float ts, int M,
                                     int N, int split, int dtype, int epi) {
  const int64_t total4 = static_cast<int64_t>(M) * N / 4;
  const int64_t plane = static_cast<int64_t>(M) * N;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 acc = reinterpret_cast<const float4*>(ws)[i];
    for (int z = 1; z < split; ++z) {
      const float4 v = reinterpret_cast<const float4*>(ws + z * plane)[i];
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const int n = static_cast<int>((i * 4) % N);
    const float o[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      store_out(out, i * 4 + j, apply_epilogue(o[j] * ts, epi, bias, n + j), dtype);
  }
}

}  // namespace bd
