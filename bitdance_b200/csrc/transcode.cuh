// transcode.cuh -- the NVFP4 -> MXFP6 transcode as device functions, plus the standalone
// global -> global transcode kernel and the operand layout kernels.
//
// The transcode rule (reference scimg/bitdance):
//   E4M3 scale byte -> (mantissa bits mb, exponent), subnormals renormalised
//                                                   (kernel/transcode_lut.py:61-76)
//   bump = mb != 0; e = exponent + bump; E8M0 = e + 127      (kernel/nvfp4_codec.py:66-70)
//   E2M3 = sign<<5 | CODE_LUT[mb][|e2m1|]                   (kernel/nvfp4_codec.py:72-75)
// With per-16 scales the two 16-blocks of a 32-block share E8M0 = max(e0, e1) + 127 and
// each folds its own mantissa with relative exponent d = emax - e_i (pair table).
//
// One 16-block = 8 packed bytes = two 32-bit words of nibbles. Magnitudes come from a
// byte-permute (prmt) over the 8-byte magnitude table of the block's (mb, d) class: one
// prmt turns four nibble selectors into four output bytes.
#pragma once
#include <cstdint>
#include "sm100.cuh"
#include "transcode_lut.cuh"

namespace bd {

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Four E2M1 nibbles (x[15:0]) -> four E2M3 code bytes (sign at bit 5).
// prmt with the nibble as selector: bit 3 (the E2M1 sign) asks for the selected byte's
// msb replicated, so a table of 0x80 bytes yields 0x80 (+) / 0xFF (-); bit 5 of that is the
// sign in E2M3 position.
__device__ __forceinline__ uint32_t nib4_to_e2m3(uint32_t x, uint32_t lo, uint32_t hi) {
  const uint32_t mag = prmt(lo, hi, x & 0x7777u);
  const uint32_t sgn = prmt(0x80808080u, 0x80808080u, x);
  return mag | (sgn & 0x20202020u);
}

// Four E2M1 nibbles -> four E4M3 bytes carrying the same MXFP6 values (E2M3 values are
// exactly representable in E4M3). A table of 0x01 bytes yields 0x01 (+) / 0x00 (-); moved
// to bit 7 it flips the sign bit that the OR set.
__device__ __forceinline__ uint32_t nib4_to_e4m3(uint32_t x, uint32_t lo, uint32_t hi) {
  const uint32_t mag = prmt(lo, hi, x & 0x7777u);
  const uint32_t pos = prmt(0x01010101u, 0x01010101u, x);
  return (mag | 0x80808080u) ^ (pos << 7);
}

// Scale-byte class table: kScaleInfo[byte & 0x7F] = (e + 16) << 3 | mb, e = exponent + bump.
struct ScaleInfoTable {
  uint8_t v[128];
};
__host__ __device__ constexpr ScaleInfoTable make_scale_info() {
  ScaleInfoTable t{};
  for (int b = 0; b < 128; ++b) {
    const int eb = (b >> 3) & 15, k = b & 7;
    int mb = 0, ex = 0;
    if (eb == 0) {
      mb = kSubMantBits[k];
      ex = kSubExp[k];
    } else {
      mb = k;
      ex = eb - 7;
    }
    const int e = ex + (mb != 0 ? 1 : 0);
    t.v[b] = static_cast<uint8_t>(((e + 16) << 3) | mb);
  }
  return t;
}

struct PermTable {
  uint32_t w[128];
};
__host__ __device__ constexpr PermTable make_perm(bool e4m3) {
  PermTable t{};
  for (int i = 0; i < 128; ++i) t.w[i] = e4m3 ? kPermE4M3[i] : kPermE2M3[i];
  return t;
}

// Shared-memory copies of the tables (filled by every kernel that transcodes).
struct alignas(16) TranscodeTables {
  uint2 perm[64];       // (d*8 + mb) -> 8 magnitude bytes
  uint8_t info[128];    // scale byte class
};
static_assert(sizeof(TranscodeTables) == 640, "tables copied as 40 16-byte words");

__host__ __device__ constexpr TranscodeTables make_tables(bool e4m3) {
  TranscodeTables t{};
  const PermTable p = make_perm(e4m3);
  // stored d-major: a warp's lookups are mostly d in {0, 1}, whose 16 rows then fall in 16
  // different bank pairs
  for (int mb = 0; mb < 8; ++mb)
    for (int d = 0; d < 8; ++d) {
      const int i = mb * 8 + d;
      t.perm[d * 8 + mb] = uint2{p.w[2 * i], p.w[2 * i + 1]};
    }
  const ScaleInfoTable s = make_scale_info();
  for (int i = 0; i < 128; ++i) t.info[i] = s.v[i];
  return t;
}

// The tables live in global memory and are copied with one coalesced 16-byte load per
// thread: per-thread-divergent reads of __constant__ data serialise within a warp, which at
// kernel start (cold constant cache) cost microseconds.
__device__ const TranscodeTables g_tables_e2m3 = make_tables(false);
__device__ const TranscodeTables g_tables_e4m3 = make_tables(true);

template <bool kE4M3>
__device__ __forceinline__ void load_tables(TranscodeTables& t, int tid, int nthreads) {
  const uint4* src = reinterpret_cast<const uint4*>(kE4M3 ? &g_tables_e4m3 : &g_tables_e2m3);
  uint4* dst = reinterpret_cast<uint4*>(&t);
  for (int i = tid; i < static_cast<int>(sizeof(TranscodeTables) / 16); i += nthreads)
    dst[i] = __ldg(src + i);
}

// Scale pair -> (table rows for each half, E8M0 byte).
__device__ __forceinline__ void scale_pair(const TranscodeTables& t, uint32_t s0, uint32_t s1,
                                           uint2& T0, uint2& T1, uint32_t& e8m0) {
  const uint32_t i0 = t.info[s0 & 0x7Fu], i1 = t.info[s1 & 0x7Fu];
  const int e0 = static_cast<int>(i0 >> 3), e1 = static_cast<int>(i1 >> 3);
  const int emax = max(e0, e1);
  const int d0 = min(emax - e0, 7), d1 = min(emax - e1, 7);
  T0 = t.perm[static_cast<uint32_t>(d0) * 8u + (i0 & 7u)];
  T1 = t.perm[static_cast<uint32_t>(d1) * 8u + (i1 & 7u)];
  e8m0 = static_cast<uint32_t>(emax + 111);  // (e + 16) - 16 + 127
}

// 32 nibbles (q) -> 32 output bytes (o0: elements 0..15, o1: 16..31).
template <bool kE4M3>
__device__ __forceinline__ void transcode32(const uint4& q, const uint2& T0, const uint2& T1,
                                            uint4& o0, uint4& o1) {
  if constexpr (kE4M3) {
    o0 = make_uint4(nib4_to_e4m3(q.x, T0.x, T0.y), nib4_to_e4m3(q.x >> 16, T0.x, T0.y),
                    nib4_to_e4m3(q.y, T0.x, T0.y), nib4_to_e4m3(q.y >> 16, T0.x, T0.y));
    o1 = make_uint4(nib4_to_e4m3(q.z, T1.x, T1.y), nib4_to_e4m3(q.z >> 16, T1.x, T1.y),
                    nib4_to_e4m3(q.w, T1.x, T1.y), nib4_to_e4m3(q.w >> 16, T1.x, T1.y));
  } else {
    o0 = make_uint4(nib4_to_e2m3(q.x, T0.x, T0.y), nib4_to_e2m3(q.x >> 16, T0.x, T0.y),
                    nib4_to_e2m3(q.y, T0.x, T0.y), nib4_to_e2m3(q.y >> 16, T0.x, T0.y));
    o1 = make_uint4(nib4_to_e2m3(q.z, T1.x, T1.y), nib4_to_e2m3(q.z >> 16, T1.x, T1.y),
                    nib4_to_e2m3(q.w, T1.x, T1.y), nib4_to_e2m3(q.w >> 16, T1.x, T1.y));
  }
}

__device__ __forceinline__ uint4 ld_stream_u4(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_stream_u4(uint4* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// ---------------------------------------------------------------------------------------
// Standalone transcode: natural layouts, one thread per 32-block, grid-stride.
template <int kScaleBlock>
__global__ void __launch_bounds__(256) transcode_kernel(const uint4* __restrict__ codes,
                                                        const uint8_t* __restrict__ scales,
                                                        uint4* __restrict__ e2m3,
                                                        uint8_t* __restrict__ e8m0,
                                                        int64_t nblk) {
  __shared__ TranscodeTables tab;
  load_tables<false>(tab, threadIdx.x, blockDim.x);
  __syncthreads();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < nblk;
       b += stride) {
    const uint4 q = ld_stream_u4(codes + b);
    uint32_t s0, s1;
    if constexpr (kScaleBlock == 16) {
      const uint32_t s = reinterpret_cast<const uint16_t*>(scales)[b];
      s0 = s & 0xFFu;
      s1 = s >> 8;
    } else {
      s0 = s1 = scales[b];
    }
    uint2 T0, T1;
    uint32_t e8;
    scale_pair(tab, s0, s1, T0, T1, e8);
    uint4 o0, o1;
    transcode32<false>(q, T0, T1, o0, o1);
    st_stream_u4(e2m3 + 2 * b, o0);
    st_stream_u4(e2m3 + 2 * b + 1, o1);
    e8m0[b] = static_cast<uint8_t>(e8);
  }
}

// ---------------------------------------------------------------------------------------
// Layout kernels.

// Natural B -> tiled: one thread per (row, 128-wide K chunk): 64 code bytes + 8 scale bytes.
__global__ void pack_b_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ sc,
                              uint8_t* __restrict__ tcodes, uint8_t* __restrict__ tsc, int N,
                              int K) {
  const int nkt = K / 128;
  const int64_t total = static_cast<int64_t>(N) * nkt;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / nkt), kc = static_cast<int>(i % nkt);
    const int64_t tile = static_cast<int64_t>(row / 128) * nkt + kc;
    const int r = row % 128;
    const uint4* src = reinterpret_cast<const uint4*>(codes + static_cast<int64_t>(row) * (K / 2) +
                                                      kc * 64);
    uint4* dst = reinterpret_cast<uint4*>(tcodes + tile * 8192 + r * 64);
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = src[j];
    const uint2 s = *reinterpret_cast<const uint2*>(sc + static_cast<int64_t>(row) * (K / 16) +
                                                    kc * 8);
    *reinterpret_cast<uint2*>(tsc + tile * 1024 + r * 8) = s;
  }
}

// Natural A codes (one per byte) -> 12+4 packed chunks; one thread per 16-element chunk.
__global__ void pack_a_codes_kernel(const uint8_t* __restrict__ codes, uint8_t* __restrict__ out,
                                    int64_t nchunks) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nchunks;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint4 v = reinterpret_cast<const uint4*>(codes)[i];
    reinterpret_cast<uint4*>(out)[i] = make_uint4(v.x & 0x3F3F3F3Fu, v.y & 0x3F3F3F3Fu,
                                                  v.z & 0x3F3F3F3Fu, v.w & 0x3F3F3F3Fu);
  }
}

// Natural A scales (M, K/32) -> [K/128][Mp4][4]; padding rows get 127.
__global__ void pack_a_scales_kernel(const uint8_t* __restrict__ e8m0, uint8_t* __restrict__ out,
                                     int M, int Mp4, int K) {
  const int nkt = K / 128;
  const int64_t total = static_cast<int64_t>(nkt) * Mp4;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int kc = static_cast<int>(i / Mp4), m = static_cast<int>(i % Mp4);
    uint32_t word = 0x7F7F7F7Fu;
    if (m < M) {
      const uint8_t* s = e8m0 + static_cast<int64_t>(m) * (K / 32) + kc * 4;
      word = static_cast<uint32_t>(s[0]) | (static_cast<uint32_t>(s[1]) << 8) |
             (static_cast<uint32_t>(s[2]) << 16) | (static_cast<uint32_t>(s[3]) << 24);
    }
    reinterpret_cast<uint32_t*>(out)[i] = word;
  }
}

// ---------------------------------------------------------------------------------------
// MXFP6 activation quantiser: fp32 / bf16 (M, K) -> E2M3 codes (M, K), one code per byte (the
// GEMM's A layout as it stands) + E8M0 per 32-block, natural (M, K/32) and/or tiled for the GEMM
// ([K/128][Mp4][4], padding rows 127).
//
// Rule (the reference's quantize(x, E8M0, E2M3), vector_quant_error.py:283-319): the block
// exponent e is the smallest integer in [-40, 40] with 7.5 * 2^e >= amax (a zero block gets
// e = 0); each element x / 2^e goes to the nearest E2M3 magnitude, an exact tie to the lower
// one (argmin keeps the first minimum, :255-280); the sign bit is set for negative elements
// whose magnitude code is not 0. With amax = m * 2^E (m in [1, 2)), 7.5 * 2^e = 1.875 * 2^(e+2),
// so e = E - 2 + (m > 1.875). E2M3 magnitudes are k/8 below 2, 2 + k/4 below 4 and 4 + k/2
// up to 7.5, so the nearest index with ties down is ceil(t - 0.5) of the scaled offset t.
// Every step is exact in fp32 (power-of-two scaling; y - 2 and y - 4 by Sterbenz; t - 0.5 for
// t >= 0.5 stays on t's grid, and t < 0.5 lands in [-0.5, 0) where the ceiling is 0 anyway),
// so the codes equal the fp64 reference's.
__device__ __forceinline__ uint32_t e2m3_code(float v, float inv_scale) {
  const float y = fminf(fabsf(v) * inv_scale, 8.0f);
  uint32_t idx;
  if (y < 2.0f) {
    idx = static_cast<uint32_t>(ceilf(y * 8.0f - 0.5f));
  } else if (y < 4.0f) {
    idx = 16u + static_cast<uint32_t>(ceilf((y - 2.0f) * 4.0f - 0.5f));
  } else {
    idx = min(31u, 24u + static_cast<uint32_t>(ceilf((y - 4.0f) * 2.0f - 0.5f)));
  }
  return idx | ((v < 0.0f && idx != 0u) ? 0x20u : 0u);
}

// Block exponent for a block amax >= 0 (see above), clamped to the E8M0 book's [-40, 40].
__device__ __forceinline__ int mxfp6_block_exp(float amax) {
  if (!(amax > 0.0f)) return 0;
  const uint32_t bits = __float_as_uint(amax);
  int E = static_cast<int>((bits >> 23) & 0xFFu) - 127;
  uint32_t frac = bits & 0x7FFFFFu;
  if (E == -127) {  // subnormal: normalise the fraction
    const int sh = __clz(static_cast<int>(frac)) - 8;
    frac = (frac << sh) & 0x7FFFFFu;
    E = -126 - sh;
  }
  const int e = E - 2 + (frac > 0x700000u ? 1 : 0);
  return max(-40, min(40, e));
}

// One warp takes 32 consecutive 16-byte vectors per step (coalesced); the lanes holding one
// 32-block (8 lanes for fp32, 4 for bf16) reduce its amax with shuffles. kUnroll steps are
// loaded before any is processed, to keep several loads in flight per lane.
template <bool kBf16>
__global__ void __launch_bounds__(256) quantize_a_kernel(const uint4* __restrict__ x,
                                                         uint8_t* __restrict__ codes,
                                                         uint8_t* __restrict__ e8m0,
                                                         uint8_t* __restrict__ scales_tiled,
                                                         int M, int K, int Mp4, uint32_t* err) {
  constexpr int kEl = kBf16 ? 8 : 4;  // elements per 16-byte vector
  constexpr int kVpb = 32 / kEl;      // vectors per 32-block
  constexpr int kUnroll = 4;
  const int64_t nvec = static_cast<int64_t>(M) * K / kEl;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int kb32 = K / 32;
  bool bad = false;
  for (int64_t base = warp * 32 * kUnroll; base < nvec; base += nwarps * 32 * kUnroll) {
    uint4 w[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = base + u * 32 + lane;
      w[u] = v < nvec ? ld_stream_u4(x + v) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = base + u * 32 + lane;
      const uint32_t ws[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
      float f[kEl];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (kBf16) {
          f[2 * j] = __uint_as_float(ws[j] << 16);
          f[2 * j + 1] = __uint_as_float(ws[j] & 0xFFFF0000u);
        } else {
          f[j] = __uint_as_float(ws[j]);
        }
      }
      float amax = 0.0f;
#pragma unroll
      for (int j = 0; j < kEl; ++j) {
        bad |= (__float_as_uint(f[j]) & 0x7F800000u) == 0x7F800000u;
        amax = fmaxf(amax, fabsf(f[j]));
      }
#pragma unroll
      for (int off = 1; off < kVpb; off <<= 1)
        amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, off));
      const int e = mxfp6_block_exp(amax);
      const float inv_scale = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e
      if (v < nvec) {
        if constexpr (kBf16) {
          uint2 o;
          o.x = e2m3_code(f[0], inv_scale) | (e2m3_code(f[1], inv_scale) << 8) |
                (e2m3_code(f[2], inv_scale) << 16) | (e2m3_code(f[3], inv_scale) << 24);
          o.y = e2m3_code(f[4], inv_scale) | (e2m3_code(f[5], inv_scale) << 8) |
                (e2m3_code(f[6], inv_scale) << 16) | (e2m3_code(f[7], inv_scale) << 24);
          reinterpret_cast<uint2*>(codes)[v] = o;
        } else {
          reinterpret_cast<uint32_t*>(codes)[v] =
              e2m3_code(f[0], inv_scale) | (e2m3_code(f[1], inv_scale) << 8) |
              (e2m3_code(f[2], inv_scale) << 16) | (e2m3_code(f[3], inv_scale) << 24);
        }
        if ((lane % kVpb) == 0) {
          const int64_t blk = v / kVpb;
          const uint8_t byte = static_cast<uint8_t>(e + 127);
          if (e8m0 != nullptr) e8m0[blk] = byte;
          if (scales_tiled != nullptr) {
            const int64_t m = blk / kb32;
            const int j = static_cast<int>(blk % kb32);
            scales_tiled[((static_cast<int64_t>(j >> 2) * Mp4 + m) << 2) + (j & 3)] = byte;
          }
        }
      }
    }
  }
  if (scales_tiled != nullptr && Mp4 > M) {  // padding rows of the tiled scales
    const int pad = Mp4 - M;
    const int64_t total = static_cast<int64_t>(K / 128) * pad;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t kc = i / pad;
      const int m = M + static_cast<int>(i % pad);
      reinterpret_cast<uint32_t*>(scales_tiled)[kc * Mp4 + m] = 0x7F7F7F7Fu;
    }
  }
  if (bad) atomicOr(err, kErrNonFinite);
}

}  // namespace bd
