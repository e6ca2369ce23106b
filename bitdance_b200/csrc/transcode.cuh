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

}  // namespace bd
