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
#include <cuda_bf16.h>

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

// 32 nibbles (q) -> 32 E2M3 code bytes (o0: elements 0..15, o1: 16..31).
__device__ __forceinline__ void transcode32(const uint4& q, const uint2& T0, const uint2& T1,
                                            uint4& o0, uint4& o1) {
  o0 = make_uint4(nib4_to_e2m3(q.x, T0.x, T0.y), nib4_to_e2m3(q.x >> 16, T0.x, T0.y),
                  nib4_to_e2m3(q.y, T0.x, T0.y), nib4_to_e2m3(q.y >> 16, T0.x, T0.y));
  o1 = make_uint4(nib4_to_e2m3(q.z, T1.x, T1.y), nib4_to_e2m3(q.z >> 16, T1.x, T1.y),
                  nib4_to_e2m3(q.w, T1.x, T1.y), nib4_to_e2m3(q.w >> 16, T1.x, T1.y));
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
// Standalone transcode: natural layouts, one consumer lane per 32-block. A CTA is 8 consumer
// warps and a producer warp whose lane 0 streams stages of 256 blocks' packed codes (4 KB,
// contiguous) into a shared-memory ring with bulk copies; lane t converts block t of each
// stage (its 16 bytes are read conflict-free) and loads the block's scale bytes from global
// memory itself, before it waits for the stage. A stage is released after the codes converted
// from it are stored (the stores depend on every word read from it).
constexpr int kTxConsumerWarps = 8;
constexpr int kTxThreads = 32 * (kTxConsumerWarps + 1);
constexpr int kTxBlocks = 32 * kTxConsumerWarps;  // blocks per stage
constexpr int kTxStageBytes = kTxBlocks * 16;
constexpr int kTxStages = 6;

template <int kScaleBlock>
__global__ void __launch_bounds__(kTxThreads, 4) transcode_kernel(const uint8_t* __restrict__ codes,
                                                                 const uint8_t* __restrict__ scales,
                                                                 uint4* __restrict__ e2m3,
                                                                 uint8_t* __restrict__ e8m0,
                                                                 int64_t nblk, uint32_t* err) {
  __shared__ TranscodeTables tab;
  __shared__ __align__(128) uint8_t stage[kTxStages][kTxStageBytes];
  __shared__ __align__(8) uint64_t full[kTxStages], empty[kTxStages];
  __shared__ uint32_t abort_word;
  volatile uint32_t* abort_flag = &abort_word;
  load_tables<false>(tab, threadIdx.x, blockDim.x);
  if (threadIdx.x == 0) {
    abort_word = 0;
    for (int i = 0; i < kTxStages; ++i) {
      mbar_init(smem_u32(&full[i]), 1);
      mbar_init(smem_u32(&empty[i]), kTxConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t nstage = (nblk + kTxBlocks - 1) / kTxBlocks;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == kTxConsumerWarps) {
    if (lane == 0) {
      int64_t i = 0;
      for (int64_t s = blockIdx.x; s < nstage; s += gridDim.x, ++i) {
        const int slot = static_cast<int>(i % kTxStages);
        const uint32_t ph = static_cast<uint32_t>(i / kTxStages) & 1u;
        if (!mbar_wait(smem_u32(&empty[slot]), ph ^ 1u, err, kErrWaitEmpty, abort_flag)) break;
        const int64_t left = nblk - s * kTxBlocks;
        const uint32_t bytes = static_cast<uint32_t>(left < kTxBlocks ? left : kTxBlocks) * 16u;
        mbar_arrive_expect_tx(smem_u32(&full[slot]), bytes);
        bulk_load(smem_u32(stage[slot]), codes + s * kTxStageBytes, bytes, smem_u32(&full[slot]));
      }
      // every copy issued has landed before the CTA exits: the last phase of each slot used
      for (int64_t j = (i > kTxStages ? i - kTxStages : 0); j < i; ++j)
        mbar_wait(smem_u32(&full[j % kTxStages]), static_cast<uint32_t>(j / kTxStages) & 1u,
                  err, kErrWaitTma, nullptr);
    }
  } else {
    const int t = threadIdx.x;
    int64_t i = 0;
    for (int64_t s = blockIdx.x; s < nstage; s += gridDim.x, ++i) {
      const int slot = static_cast<int>(i % kTxStages);
      const uint32_t ph = static_cast<uint32_t>(i / kTxStages) & 1u;
      const int64_t b = s * kTxBlocks + t;
      const bool valid = b < nblk;
      uint32_t sc = 0;
      if (valid) {
        if constexpr (kScaleBlock == 16)
          sc = reinterpret_cast<const uint16_t*>(scales)[b];
        else
          sc = scales[b];
      }
      if (!mbar_wait(smem_u32(&full[slot]), ph, err, kErrWaitTma, abort_flag)) break;
      if (valid) {
        const uint4 q = reinterpret_cast<const uint4*>(stage[slot])[t];
        uint32_t s0, s1;
        if constexpr (kScaleBlock == 16) {
          s0 = sc & 0xFFu;
          s1 = sc >> 8;
        } else {
          s0 = s1 = sc;
        }
        uint2 T0, T1;
        uint32_t e8;
        scale_pair(tab, s0, s1, T0, T1, e8);
        uint4 o0, o1;
        transcode32(q, T0, T1, o0, o1);
        st_stream_u4(e2m3 + 2 * b, o0);
        st_stream_u4(e2m3 + 2 * b + 1, o1);
        e8m0[b] = static_cast<uint8_t>(e8);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty[slot]));
    }
  }
}

// ---------------------------------------------------------------------------------------
// Layout kernels.

// The weights are static, so the tiled layout the GEMM reads carries the parts of the transcode
// that depend on them alone, prepared once here:
//  * code words: in each 32-bit word of E2M1 codes (elements 0..7 in nibbles 0..7) the
//    magnitudes stay in nibble bits 0..2 and the sign of element i moves to bit 8i + 7 (i < 4)
//    or 8(i - 4) + 3 (i >= 4), where an E4M3 byte of the low or (shifted by 4) high output word
//    carries it;
//  * per 32-block a 16-bit class word instead of the two E4M3 scale bytes (same size), from the
//    scale-byte classes c = (e + 16) << 3 | mb (e = exponent + bump, 7..25; the info table):
//    bits 0..5 the magnitude-table row d*8 + mb of the 16-block with the smaller e (d = the
//    exponent gap, at most 7), bits 6..8 the mantissa bits of the other (its row, d = 0), bit 9
//    set when that other one is the first 16-block, bits 10..14 emax - 7 (E8M0 = field + 118).
__host__ __device__ constexpr uint32_t sign_spread(uint32_t w) {
  uint32_t r = w & 0x77777777u;
  for (int i = 0; i < 8; ++i)
    r |= ((w >> (4 * i + 3)) & 1u) << (i < 4 ? 8 * i + 7 : 8 * (i - 4) + 3);
  return r;
}
__host__ __device__ constexpr uint32_t pair_sideband(uint32_t c0, uint32_t c1) {
  const uint32_t e0 = c0 >> 3, e1 = c1 >> 3;
  const uint32_t first_big = e0 > e1 ? 1u : 0u;
  const uint32_t em = first_big ? e0 : e1, es = first_big ? e1 : e0;
  const uint32_t d = em - es < 7u ? em - es : 7u;
  const uint32_t small_row = d * 8u + ((first_big ? c1 : c0) & 7u);
  const uint32_t big_mb = (first_big ? c0 : c1) & 7u;
  return small_row | (big_mb << 6) | (first_big << 9) | ((em - 7u) << 10);
}

// Natural B -> tiled: one thread per (row, 128-wide K chunk): 64 code bytes + 8 scale bytes,
// transcode-ready (kClassWords) or only regrouped (the E4M3 sideband).
template <bool kClassWords>
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
    uint2* sdst = reinterpret_cast<uint2*>(tsc + tile * 1024 + r * 8);
    const uint8_t* s = sc + static_cast<int64_t>(row) * (K / 16) + kc * 8;
    if constexpr (!kClassWords) {
#pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = src[j];
      *sdst = *reinterpret_cast<const uint2*>(s);
      continue;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = src[j];
      dst[j] = make_uint4(sign_spread(v.x), sign_spread(v.y), sign_spread(v.z), sign_spread(v.w));
    }
    uint32_t f[4];
#pragma unroll
    for (int b = 0; b < 4; ++b)
      f[b] = pair_sideband(g_tables_e4m3.info[s[2 * b] & 0x7Fu],
                           g_tables_e4m3.info[s[2 * b + 1] & 0x7Fu]);
    *sdst = make_uint2(f[0] | (f[1] << 16), f[2] | (f[3] << 16));
  }
}

// Natural A codes (one per byte) -> 12+4 packed chunks; one thread per 16-element chunk.
// MXFP4 weight scales -> the E4M3 sideband: E8M0 byte e of a 32-block becomes, for both of
// its 16-blocks, the E4M3 byte of the same power of two 2^(e - 127) (normal for exponents
// -6..8, subnormal 0x04 / 0x02 / 0x01 for -7 / -8 / -9). With a power-of-two E4M3 scale the
// pair rule reproduces the MXFP4 block exactly (mantissa bits 0: no bump, codes = the E2M1
// magnitudes, E8M0 = e), so an MXFP4 weight (the reference's "w4a6" arm: E2M1 codes with E8M0
// per-32 scales) runs through the NVFP4 GEMM unchanged. Exponents outside -9..8 have no E4M3
// form: the block's scale becomes 0 and kErrRange is raised in the error word.
__global__ void e8m0_to_e4m3_pairs_kernel(const uint8_t* __restrict__ e8m0,
                                          uint16_t* __restrict__ pairs, int64_t n,
                                          uint32_t* err) {
  bool bad = false;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(e8m0[i]) - 127;
    uint32_t b;
    if (s >= -6 && s <= 8) b = static_cast<uint32_t>(s + 7) << 3;
    else if (s >= -9) b = 0x04u >> (-7 - s);  // -7, -8, -9: subnormal 2^-7, 2^-8, 2^-9
    else {
      b = 0u;
      bad = true;
    }
    pairs[i] = static_cast<uint16_t>(b | (b << 8));
  }
  if (bad) atomicOr(err, kErrRange);
}

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
// whose magnitude code is not 0.
//
// Block exponent: with amax = m * 2^E (m in [1, 2)), 7.5 * 2^e = 1.875 * 2^(e+2), so
// e = E - 2 + (m > 1.875); every amax below 2^-38 (subnormals included) clamps to -40.
//
// Element code, integer arithmetic on float bits (no conversions): for y = |x| / 2^e >= 1 the
// E2M3 index is (exponent field - 126) * 8 + top three mantissa bits, rounded up when the 20
// bits below them are strictly above half -- adding 0x7FFFF carries into bit 20 exactly then,
// and a carry out of the mantissa moves to the next binade as the index does; so
// idx = ((bits(y) + 0x7FFFF) >> 20) - 1008, capped at 31. For y < 1 (E2M3 subnormals, step 1/8)
// the same formula applied to z = (y + 1) / 2 in [0.5, 1) gives round-half-down(8 y): z's
// mantissa is y's binary expansion, and rounding z UP to float keeps the "strictly above half"
// decision (a truncated remainder r with lost low bits is above half exactly when r >= half,
// exactly when r + 1 ulp > half). z <= y for y >= 1 and z > y for y < 1, so max(y, z) picks
// the right operand with no compare. y = |x| * 2^-e is exact (an exponent shift; values that
// leave the normal range are far below 1/16 and map to code 0 either way).
__device__ __forceinline__ uint32_t e2m3_mag(float v, float inv_scale) {
  const float y = fabsf(v) * inv_scale;
  const float z = __fmaf_ru(y, 0.5f, 0.5f);
  const uint32_t t = __float_as_uint(fmaxf(y, z));
  return min((t + (0x7FFFFu - (1008u << 20))) >> 20, 31u);
}

// The same index left in bits 24..28 of the result (byte 3, so that byte permutes pack four of
// them) for y <= 7.75, where (bits + 0x7FFFF - (1008 << 20)) mod 2^32 < 2^25: one multiply-add,
// 16 * bits + 16 * (0x7FFFF - (1008 << 20)) mod 2^32. The block exponent keeps y <= 7.5 except
// when it is clamped at 40; that case takes e2m3_mag.
__device__ __forceinline__ uint32_t e2m3_mag_b3(float v, float inv_scale) {
  const float y = fabsf(v) * inv_scale;
  const float z = __fmaf_ru(y, 0.5f, 0.5f);
  return __float_as_uint(fmaxf(y, z)) * 16u + 0x107FFFF0u;
}

// Byte 3 of each of four words -> one word (three byte permutes).
__device__ __forceinline__ uint32_t gather_b3(uint32_t x0, uint32_t x1, uint32_t x2, uint32_t x3) {
  return prmt(prmt(x0, x1, 0x0073u), prmt(x2, x3, 0x7300u), 0x7610u);
}

// 4 magnitude codes (bytes, each <= 31) + 0xFF sign bytes of the negative elements -> 4 E2M3
// codes; the sign (bit 5) is kept only on non-zero codes: for a byte b <= 31, b + 31 has bit 5
// set exactly when b >= 1, with no carry between bytes.
__device__ __forceinline__ uint32_t e2m3_word(uint32_t mags, uint32_t neg) {
  return mags | ((mags + 0x1F1F1F1Fu) & neg & 0x20202020u);
}

__device__ __forceinline__ uint32_t pack4(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3) {
  return c0 | (c1 << 8) | (c2 << 16) | (c3 << 24);
}

// max(a, b) that returns NaN when either is NaN.
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Block exponent from the bits of the block amax (finite, sign cleared).
__device__ __forceinline__ int mxfp6_block_exp(uint32_t amax_bits) {
  if (amax_bits == 0u) return 0;
  const int E = static_cast<int>(amax_bits >> 23) - 127;
  const int e = E - 2 + ((amax_bits & 0x7FFFFFu) > 0x700000u ? 1 : 0);
  return max(-40, min(40, e));
}

// Codes of 4 elements (fp32 values) with the block's 2^-e; `clamp` for blocks whose exponent
// was clamped at 40 (elements may exceed 7.5 there).
__device__ __forceinline__ uint32_t e2m3_mags4(float f0, float f1, float f2, float f3, float inv,
                                               bool clamp) {
  if (!clamp)
    return gather_b3(e2m3_mag_b3(f0, inv), e2m3_mag_b3(f1, inv), e2m3_mag_b3(f2, inv),
                     e2m3_mag_b3(f3, inv));
  return pack4(e2m3_mag(f0, inv), e2m3_mag(f1, inv), e2m3_mag(f2, inv), e2m3_mag(f3, inv));
}

// Stage geometry of the quantiser. One consumer lane owns one 32-element block per stage: a
// CTA is kQConsumerWarps consumer warps (256 lanes) plus one producer warp whose lane 0 loads
// stages of 256 blocks into a shared-memory ring with 2-D tensor copies (completion on
// mbarrier tx-counts), so loads stay in flight while the consumers compute. A block is one
// swizzled shared-memory row (64 bytes of bf16 with the 64-byte swizzle, 128 bytes of fp32
// with the 128-byte swizzle): lane t reads 16-byte chunk c of row t at chunk c ^ swz(t), and
// the eight lanes of each shared-memory phase then cover all 32 banks.
constexpr int kQConsumerWarps = 8;
constexpr int kQThreads = 32 * (kQConsumerWarps + 1);
constexpr int kQRows = 32 * kQConsumerWarps;  // blocks per stage

template <bool kBf16>
struct QuantCfg {
  static constexpr int kRowBytes = kBf16 ? 64 : 128;
  static constexpr int kChunks = kRowBytes / 16;
  static constexpr int kStageBytes = kQRows * kRowBytes;  // 16 KB / 32 KB
  static constexpr int kStages = kBf16 ? 4 : 3;
  static constexpr int kCtasPerSm = kBf16 ? 3 : 2;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;  // + alignment slack
  // chunk index bits XORed by the swizzle: address bits [5:4] ^= [8:7] (64-byte mode),
  // [6:4] ^= [9:7] (128-byte mode), with rows of kRowBytes from a 1 KB aligned base
  __device__ static __forceinline__ int swz(int row) { return kBf16 ? (row >> 1) & 3 : row & 7; }
};

// Quantise the 32-block in chunks q[] (its natural order): codes into 8 words o[], returns the
// E8M0 byte; `bad` set when the block holds an Inf or NaN.
template <bool kBf16>
__device__ __forceinline__ uint32_t quantize_block(const uint4 (&q)[QuantCfg<kBf16>::kChunks],
                                                   uint32_t (&o)[8], bool& bad) {
  constexpr int kC = QuantCfg<kBf16>::kChunks;
  // block amax, NaN-propagating (an Inf or NaN anywhere makes it non-finite); bf16 pairs are
  // compared two at a time
  float am = 0.0f;
  if constexpr (kBf16) {
    __nv_bfloat162 m2 = __habs2(*reinterpret_cast<const __nv_bfloat162*>(&q[0].x));
#pragma unroll
    for (int c = 0; c < kC; ++c) {
      const uint32_t ws[4] = {q[c].x, q[c].y, q[c].z, q[c].w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        m2 = __hmax2_nan(m2, __habs2(*reinterpret_cast<const __nv_bfloat162*>(&ws[j])));
    }
    const uint32_t mb = *reinterpret_cast<const uint32_t*>(&m2);
    am = fmax_nan(__uint_as_float(mb << 16), __uint_as_float(mb & 0xFFFF0000u));
  } else {
#pragma unroll
    for (int c = 0; c < kC; ++c) {
      am = fmax_nan(am, fabsf(__uint_as_float(q[c].x)));
      am = fmax_nan(am, fabsf(__uint_as_float(q[c].y)));
      am = fmax_nan(am, fabsf(__uint_as_float(q[c].z)));
      am = fmax_nan(am, fabsf(__uint_as_float(q[c].w)));
    }
  }
  const uint32_t amax = __float_as_uint(am);
  bad |= amax >= 0x7F800000u;  // an Inf or NaN in the block
  const int e = mxfp6_block_exp(amax);
  const float inv = __uint_as_float(static_cast<uint32_t>(127 - e) << 23);  // 2^-e
  const bool clamp = e == 40;
#pragma unroll
  for (int c = 0; c < kC; ++c) {
    const uint32_t w0 = q[c].x, w1 = q[c].y, w2 = q[c].z, w3 = q[c].w;
    if constexpr (kBf16) {
      // 0xFF sign bytes: bits 15 and 31 of each input word, replicated over the byte (a prmt
      // selector nibble with its top bit set copies the sign of the selected byte)
      o[2 * c] = e2m3_word(
          e2m3_mags4(__uint_as_float(w0 << 16), __uint_as_float(w0 & 0xFFFF0000u),
                     __uint_as_float(w1 << 16), __uint_as_float(w1 & 0xFFFF0000u), inv, clamp),
          prmt(w0, w1, 0xFDB9u));
      o[2 * c + 1] = e2m3_word(
          e2m3_mags4(__uint_as_float(w2 << 16), __uint_as_float(w2 & 0xFFFF0000u),
                     __uint_as_float(w3 << 16), __uint_as_float(w3 & 0xFFFF0000u), inv, clamp),
          prmt(w2, w3, 0xFDB9u));
    } else {
      o[c] = e2m3_word(e2m3_mags4(__uint_as_float(w0), __uint_as_float(w1), __uint_as_float(w2),
                                  __uint_as_float(w3), inv, clamp),
                       prmt(prmt(w0, w1, 0x00FBu), prmt(w2, w3, 0xFB00u), 0x7610u));
    }
  }
  return static_cast<uint32_t>(e + 127);
}

template <bool kBf16>
__global__ void __launch_bounds__(kQThreads, QuantCfg<kBf16>::kCtasPerSm)
    quantize_a_kernel(const __grid_constant__ CUtensorMap tm_x, uint8_t* __restrict__ codes,
                      uint8_t* __restrict__ e8m0, uint8_t* __restrict__ scales_tiled, int M,
                      int K, int Mp4, uint64_t nkt_magic, uint32_t* err) {
  using Cfg = QuantCfg<kBf16>;
  extern __shared__ __align__(1024) uint8_t qsm_raw[];
  uint8_t* qsm = qsm_raw + ((1024u - (smem_u32(qsm_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t full[Cfg::kStages], empty[Cfg::kStages];
  __shared__ uint32_t abort_word;
  volatile uint32_t* abort_flag = &abort_word;
  const int64_t nblk = static_cast<int64_t>(M) * (K / 32);
  const int64_t nstage = (nblk + kQRows - 1) / kQRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    abort_word = 0;
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), kQConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // a kernel launched after this one with programmatic serialisation (the GEMM that consumes
  // these codes) may be scheduled on free SMs now; it waits for this grid before reading them.
  // When this grid was itself launched that way, x and the outputs belong to the previous grid
  // until it completes (it may still be reading a recycled output buffer).
  grid_dep_launch_dependents();
  grid_dep_wait();
  if (warp == kQConsumerWarps) {
    // ---- producer: stages blockIdx.x, + gridDim.x, ... (rows of 256 blocks) into the ring;
    // a partial last stage is zero-filled past the last block and still counts the full box
    if (lane == 0) {
      prefetch_tmap(&tm_x);
      int64_t i = 0;
      for (int64_t s = blockIdx.x; s < nstage; s += gridDim.x, ++i) {
        const int slot = static_cast<int>(i % Cfg::kStages);
        const uint32_t ph = static_cast<uint32_t>(i / Cfg::kStages) & 1u;
        if (!mbar_wait(smem_u32(&empty[slot]), ph ^ 1u, err, kErrWaitEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(smem_u32(&full[slot]), Cfg::kStageBytes);
        tma_load_2d(smem_u32(qsm + slot * Cfg::kStageBytes), &tm_x, 0,
                    static_cast<int32_t>(s * kQRows), smem_u32(&full[slot]));
      }
      // every copy issued has landed before the CTA exits: the last phase of each slot used
      for (int64_t j = (i > Cfg::kStages ? i - Cfg::kStages : 0); j < i; ++j)
        mbar_wait(smem_u32(&full[j % Cfg::kStages]), static_cast<uint32_t>(j / Cfg::kStages) & 1u,
                  err, kErrWaitTma, nullptr);
    }
  } else {
    // ---- consumers: lane t of the CTA quantises block t of each stage
    const int t = threadIdx.x;
    const uint32_t nkt = static_cast<uint32_t>(K / 128);
    const int swz = Cfg::swz(t);
    bool bad = false;
    int64_t i = 0;
    for (int64_t s = blockIdx.x; s < nstage; s += gridDim.x, ++i) {
      const int slot = static_cast<int>(i % Cfg::kStages);
      const uint32_t ph = static_cast<uint32_t>(i / Cfg::kStages) & 1u;
      if (!mbar_wait(smem_u32(&full[slot]), ph, err, kErrWaitTma, abort_flag)) break;
      const uint8_t* row = qsm + slot * Cfg::kStageBytes + t * Cfg::kRowBytes;
      uint4 q[Cfg::kChunks];
#pragma unroll
      for (int c = 0; c < Cfg::kChunks; ++c)
        q[c] = *reinterpret_cast<const uint4*>(row + ((c ^ swz) << 4));
      uint32_t o[8];
      const uint32_t byte = quantize_block<kBf16>(q, o, bad);
      const int64_t b = s * kQRows + t;
      const bool valid = b < nblk;
      if (valid) {
        uint4* dst = reinterpret_cast<uint4*>(codes + b * 32);
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        if (e8m0 != nullptr) e8m0[b] = static_cast<uint8_t>(byte);
      }
      if (scales_tiled != nullptr) {
        // blocks 4j..4j+3 (one 128-element chunk of a row, K % 128 == 0) sit on lanes 4j..4j+3
        const uint32_t b1 = __shfl_down_sync(0xFFFFFFFFu, byte, 1);
        const uint32_t b2 = __shfl_down_sync(0xFFFFFFFFu, byte, 2);
        const uint32_t b3 = __shfl_down_sync(0xFFFFFFFFu, byte, 3);
        if ((lane & 3) == 0 && valid) {
          // chunk -> (row, chunk in row): chunk < 2^31 and nkt < 2^17, so the high half of
          // chunk * (floor(2^64 / nkt) + 1) is the exact quotient (nkt = 1 has no 64-bit magic)
          const uint32_t chunk = static_cast<uint32_t>(b >> 2);
          const uint32_t m =
              nkt == 1u ? chunk : static_cast<uint32_t>(__umul64hi(chunk, nkt_magic));
          const uint32_t kc = chunk - m * nkt;
          reinterpret_cast<uint32_t*>(scales_tiled)[static_cast<int64_t>(kc) * Mp4 + m] =
              pack4(byte, b1, b2, b3);
        }
      }
      // the stage is released after the codes computed from it are stored
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty[slot]));
    }
    if (scales_tiled != nullptr && Mp4 > M) {  // padding rows of the tiled scales
      const int pad = Mp4 - M;
      const int64_t ptotal = static_cast<int64_t>(K / 128) * pad;
      for (int64_t u = static_cast<int64_t>(blockIdx.x) * kQRows + t; u < ptotal;
           u += static_cast<int64_t>(gridDim.x) * kQRows) {
        const int64_t kc = u / pad;
        const int m = M + static_cast<int>(u % pad);
        reinterpret_cast<uint32_t*>(scales_tiled)[kc * Mp4 + m] = 0x7F7F7F7Fu;
      }
    }
    if (bad) atomicOr(err, kErrNonFinite);
  }
}

}  // namespace bd
