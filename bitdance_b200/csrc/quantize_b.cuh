// quantize_b.cuh -- NVFP4 weight quantiser on the GPU: fp32 / bf16 weights (N, K) -> E2M1 codes
// packed two per byte (N, K/2), one E4M3 scale byte per 16 elements (N, K/16), and the fp32
// per-tensor scale.
//
// Rule (the reference's two-level NVFP4 encode: run_method, remote/quant_real_weights.py:273-287,
// then encode_nvfp4, kernel/nvfp4_codec.py:34-63, over quantize / choose_scales /
// nearest_codes, vector_quant_error.py:255-319):
//   s_t   = float32(amax(|w|) / (448 * 6)) computed in double, 1.0 for an all-zero tensor;
//   v     = w / s_t in float32 (round to nearest);
//   per 16-block: B = the smallest E4M3FN value (normals 2^-6 .. 448; the reference's default
//         book has no subnormals) >= amax(|v|) / 6, 448 when none is, 1.0 for a zero block;
//   code  = the nearest E2M1 magnitude {0, .5, 1, 1.5, 2, 3, 4, 6} to |v| / B, an exact tie to
//         the lower one; the sign bit only on non-zero codes; the scale byte is the E4M3
//         encoding of B.
//
// Exactness without double arithmetic per element. The reference compares double quotients;
// here every comparison is between exact float32 values:
//   * B >= fl64(amax / 6)  <=>  6 B >= amax, because a float32 amax that is not exactly 6 B
//     differs from it by at least 2^-24 relative, far above the double rounding error. The
//     smallest float32 >= amax / 6 is __fdiv_ru(amax, 6), and the smallest value with a 3-bit
//     mantissa above that is it rounded up at bit 20.
//   * |v| / B > m (m an E2M1 midpoint) <=>  |v| > m * B, and m * B (at most 7 significant bits)
//     is exact in float32; the same 2^-24 argument covers the double quotient.
#pragma once
#include <cstdint>

#include <cuda_bf16.h>

#include "sm100.cuh"

namespace bd {

// Tensor amax of |w| as float bits (non-negative floats order as unsigned integers); an Inf or
// NaN anywhere sets kErrNonFinite. stat[1] must be zero before the launch.
template <bool kBf16>
__global__ void __launch_bounds__(256) weight_amax_kernel(const uint4* __restrict__ w,
                                                          int64_t nvec, uint32_t* stat,
                                                          uint32_t* err) {
  uint32_t m = 0;
  bool bad = false;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 q = w[i];
    const uint32_t ws[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (kBf16) {
        const uint32_t lo = (ws[j] << 16) & 0x7FFFFFFFu, hi = ws[j] & 0x7FFF0000u;
        bad |= lo >= 0x7F800000u || hi >= 0x7F800000u;
        m = max(m, max(lo, hi));
      } else {
        const uint32_t a = ws[j] & 0x7FFFFFFFu;
        bad |= a >= 0x7F800000u;
        m = max(m, a);
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
  if ((threadIdx.x & 31) == 0 && m != 0) atomicMax(stat + 1, m);
  if (bad) atomicOr(err, kErrNonFinite);
}

// s_t from the tensor amax bits: float32(amax / 2688) via double, 1.0 for amax == 0.
__device__ __forceinline__ float nvfp4_tensor_scale(uint32_t amax_bits) {
  if (amax_bits == 0u) return 1.0f;
  return __double2float_rn(__ddiv_rn(static_cast<double>(__uint_as_float(amax_bits)), 2688.0));
}

// E4M3 block scale for a 16-block amax (float32, >= 0): the value B and its byte.
__device__ __forceinline__ float nvfp4_block_scale(float amax, uint32_t& byte) {
  if (amax == 0.0f) {
    byte = 0x38u;  // 1.0
    return 1.0f;
  }
  uint32_t b = __float_as_uint(__fdiv_ru(amax, 6.0f));
  if (b & 0xFFFFFu) b = (b | 0xFFFFFu) + 1u;   // round up to a 3-bit mantissa
  b = max(b, 0x3C800000u);                     // >= 2^-6, the smallest normal E4M3
  b = min(b, 0x43E00000u);                     // <= 448
  const uint32_t e = (b >> 23) - 127u + 7u;    // biased E4M3 exponent, 1..15
  byte = (e << 3) | ((b >> 20) & 7u);
  return __uint_as_float(b);
}

// E2M1 code (sign << 3 | index) of a scaled element v against the block's midpoint products
// t[i] = m_i * B (m = .25 .75 1.25 1.75 2.5 3.5 5): the index counts the midpoints strictly
// below |v|, so a tie goes to the lower magnitude.
__device__ __forceinline__ uint32_t e2m1_code(float v, const float (&t)[7]) {
  const float a = fabsf(v);
  uint32_t idx = 0;
#pragma unroll
  for (int i = 0; i < 7; ++i) idx += a > t[i] ? 1u : 0u;
  return idx | ((v < 0.0f && idx != 0u) ? 8u : 0u);
}

// One thread per 16-block: 16 elements in (64 B fp32 / 32 B bf16), 8 code bytes + 1 scale byte
// out. stat[1] holds the tensor amax bits (weight_amax_kernel); block 0 writes s_t to stat[0].
template <bool kBf16>
__global__ void __launch_bounds__(256) quantize_b_kernel(const uint8_t* __restrict__ w,
                                                         uint8_t* __restrict__ codes,
                                                         uint8_t* __restrict__ scales,
                                                         int64_t nblk, uint32_t* stat) {
  const float s_t = nvfp4_tensor_scale(stat[1]);
  if (blockIdx.x == 0 && threadIdx.x == 0) reinterpret_cast<float*>(stat)[0] = s_t;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < nblk;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v[16];
    if constexpr (kBf16) {
      const uint4* src = reinterpret_cast<const uint4*>(w + b * 32);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 q = src[h];
        const uint32_t ws[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[8 * h + 2 * j] = __uint_as_float(ws[j] << 16);
          v[8 * h + 2 * j + 1] = __uint_as_float(ws[j] & 0xFFFF0000u);
        }
      }
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(w + b * 64);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint4 q = src[h];
        v[4 * h] = __uint_as_float(q.x);
        v[4 * h + 1] = __uint_as_float(q.y);
        v[4 * h + 2] = __uint_as_float(q.z);
        v[4 * h + 3] = __uint_as_float(q.w);
      }
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[j] = __fdiv_rn(v[j], s_t);
      amax = fmaxf(amax, fabsf(v[j]));
    }
    uint32_t sbyte;
    const float B = nvfp4_block_scale(amax, sbyte);
    const float t[7] = {0.25f * B, 0.75f * B, 1.25f * B, 1.75f * B, 2.5f * B, 3.5f * B, 5.0f * B};
    uint32_t word[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t x = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) x |= e2m1_code(v[8 * h + j], t) << (4 * j);
      word[h] = x;
    }
    reinterpret_cast<uint2*>(codes)[b] = make_uint2(word[0], word[1]);
    scales[b] = static_cast<uint8_t>(sbyte);
  }
}

}  // namespace bd
