// gemm.cuh -- fused W4A6 GEMM for sm_100a: C = A_mxfp6 . transcode(B_nvfp4)^T.
//
// One block-scaled tcgen05.mma (kind::mxf8f6f4, M = 128, K = 32) costs the tensor core the
// same time whatever its N (16..256), so the weights are the MMA's N operand, 256 rows per
// MMA, and the tokens are its M operand, read from tensor memory (128 lanes; a decode batch
// writes only its BM <= 128 token rows, no MMA read ever touches memory a copy may be
// writing). Output tile: BM tokens x 256 weight rows, accumulated in tensor memory as 128
// lanes (tokens) x 256 fp32 columns (weight rows).
//
// Persistent CTAs walk a schedule of "segments" (a tile and a range of 128-wide K chunks):
//   * stream-K (the default): the (tile, K chunk) units are cut into one contiguous range per
//     CTA; a tile split between CTAs is finished in-kernel -- every contributor stores its
//     fp32 partial in a per-CTA slot, the last one to arrive (atomic counter) sums the slots
//     in CTA order and writes C, so results do not depend on timing;
//   * explicit split-K (split_k >= 1): items (tile, split) dealt round-robin, written as
//     partial planes, fp32 workspace planes or fp32 atomics (the reference's split modes).
//
// Warp roles (736 threads):
//   warp 0      weight producer  TMA: packed NVFP4 codes (2 x 8 KB per chunk, 64B-swizzled)
//                                and their scale sideband (2 x 1 KB: class words, or E4M3
//                                bytes with BD_GEMM_B_E4M3) into the weight ring.
//   warp 22     token producer   TMA: token rows (one E2M3 code per byte, 128B-swizzled) and
//                                their E8M0 scales into the token ring.
//   warps 6..21 transcode        two groups of 8 warps taking alternate chunks (two chunks in
//                                flight); thread (warp gw of its group, lane l) converts the
//                                four K blocks of weight row 32 gw + l into
//                                E4M3 bytes of the 128B-swizzled operand tile in shared memory
//                                (the B ring) and stages the rows' E8M0 scales.
//   warp 1      MMA              4 block-scaled tcgen05.mma per chunk (A = tokens from tensor
//                                memory, B = transcoded weights from shared memory); its
//                                commits free the B and token slots.
//   warps 2..5  epilogue         one warp per tensor-memory lane quarter. Per chunk, for
//                                128-row token tiles: the quarter's token rows (the MMA's A
//                                operand) and the token and weight scale factors into tensor
//                                memory (tcgen05.st); decode tiles (BM <= 64) have the
//                                transcode group that converted the chunk do this itself
//                                (kGroupDelivers). Per segment: tensor-memory accumulator ->
//                                registers -> C / partials.
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

constexpr int cround(int x, int a) { return (x + a - 1) / a * a; }

constexpr int kTileN = 256;  // weight rows per tile (the MMA's N)

// Ring depths per token rows BM: weight ring SW (raw NVFP4 in shared memory, released by the
// transcode warps), B ring SB (transcoded operand, released by the MMA), token ring ST, and G,
// the number of transcode warp groups that take chunks in turn. SW and SB are multiples of G,
// so a slot is only ever used by one group, in order: no waiter can run a whole phase ahead.
// When the groups also take the token slots (kGroupDelivers), ST is a multiple of G for the
// same reason: a group waiting on a token slot has itself consumed the slot's previous fill, so
// the fill it waits for is never two phases ahead of the barrier (a parity wait would pass on
// the older phase and copy stale token rows). Decode tiles of up to 32 rows use four groups of
// four warps (two weight rows per thread): four chunks in flight, measured 2 % faster than
// two groups of eight there.
struct RingDepths {
  int sw, sb, st, groups;
};
constexpr RingDepths ring_depths(int BM) {
  // CTA-pair tiles (BM = 256, 128 token rows and 128 weight rows per CTA): four slots of each
  // ring, four groups of four warps (one weight row per thread)
  if (BM == 256) return {4, 4, 4, 4};
  if (BM <= 16) return {4, 4, 4, 4};
  if (BM <= 32) return {4, 4, 4, 4};
  if (BM <= 64) return {4, 2, 6, 2};
  // 128-row tiles: four B slots fit only with two weight and two token slots, which the
  // transcode warps and the epilogue warps release as soon as they hold the stage's words in
  // registers (kEarlyRelease)
  return {2, 4, 2, 2};
}

// BM = 256: a tile of 256 token rows x 256 weight rows computed by a cluster of two CTAs with
// the pair MMA (tcgen05 cta_group::2): CTA rank r loads, holds and stores token rows
// 128 r .. 128 r + 127 of the tile, and loads and transcodes weight rows 128 r .. 128 r + 127
// (the second operand of the MMA is split between the two CTAs' shared memory); rank 0 issues
// the MMAs. Every weight chunk is transcoded once per 256 tokens instead of once per 128.
template <int BM>
struct GemmCfg {
  static constexpr int kBM = BM;
  static constexpr bool kPair = BM == 256;
  static constexpr int kRows = kPair ? 128 : BM;   // token rows per CTA
  static constexpr int kBRows = kPair ? 128 : 256;  // weight rows per CTA (B operand rows)
  static constexpr int SW = ring_depths(BM).sw;
  static constexpr int SB = ring_depths(BM).sb;
  static constexpr int ST = ring_depths(BM).st;
  static constexpr int kGroups = ring_depths(BM).groups;  // transcode warp groups
  // weight stages released after their loads (guarded by a dependent store), token slots by
  // the epilogue warps after their copy into tensor memory; otherwise after the B rows are
  // stored and by the MMA's commit
  static constexpr bool kEarlyRelease = BM >= 128;
  // decode tiles: the transcode group that converted a chunk also writes the chunk's token rows
  // and scale factors into tensor memory and signals the MMA itself (one hand-off fewer per
  // chunk); 128-row tiles leave that to the epilogue warps (measured faster there)
  // (and CTA pairs, whose per-chunk delivery by the four epilogue warps was the bottleneck once
  // each CTA transcodes half the rows)
  static constexpr bool kGroupDelivers = BM <= 64 || kPair;
  // token ring: BM rows x 128 B per slot (one E2M3 code per byte, 128B-swizzled so the copy
  // into tensor memory reads without bank conflicts), and the BM E8M0 words of each slot in a
  // separate small ring.
  static constexpr int kTRowBytes = kRows * 128;
  static constexpr int kTScaleBytes = kRows * 4;
  static constexpr int kTScaleSlot = cround(kTScaleBytes, 128);  // TMA destinations: 128 B aligned
  static constexpr int kTTx = kTRowBytes + kTScaleBytes;
  // weight stage: the CTA's 128-row halves x (8 KB codes, 64B-swizzled), then the 1 KB scale
  // tiles of both halves of the tile (a CTA of a pair derives the peer half's E8M0 words too)
  static constexpr int kWHalves = kBRows / 128;
  static constexpr int kWCodes = 8192 * kWHalves;
  static constexpr int kWStage = kWCodes + 2048;
  // B stage: kBRows rows x 128 B E4M3 (128B-swizzled, K-major)
  static constexpr int kBStage = kBRows * 128;
  static constexpr int oT = 0;
  static constexpr int oW = ST * kTRowBytes;
  static constexpr int oB = oW + SW * kWStage;
  static constexpr int oSf = oB + SB * kBStage;  // SB x 256 E8M0 words staged for tensor memory
  // magnitude table, kPermCopies copies interleaved (entry e of copy j at e * 8 * kPermCopies
  // + j * 8), lane l reads copy l % kPermCopies. With 16 copies (decode tiles) copy j sits in
  // bank pair j whatever the row, so the 8-byte lookups of a warp take the minimum two
  // shared-memory wavefronts; 128-row tiles keep 8 copies (measured faster there), and so do
  // 32-row tiles, whose four token slots leave no room for 16.
  static constexpr int kPermCopies = (BM <= 64 && BM != 32) ? 16 : 8;
  static constexpr int kRowShift = (BM <= 64 && BM != 32) ? 7 : 6;  // log2 of a table row's stride
  static constexpr int oPerm = oSf + SB * 1024;
  static constexpr int oTs = oPerm + 64 * 8 * kPermCopies;  // token scale ring
  // 128-row tiles write C through shared memory with TMA stores (GemmParams::tma_c): per
  // epilogue warp two staging buffers of 32 rows, for CTA pairs of 128 B (64 16-bit outputs,
  // 128B-swizzled: half the stores, fences and buffer waits of a drain, prefill -1 to -2 %),
  // else of 64 B (32 outputs, 64B-swizzled; single 128-row CTAs have no room for more)
  static constexpr bool kTmaStore = BM >= 128;
  static constexpr int kCCols = kPair ? 64 : 32;  // 16-bit outputs per staging row
  static constexpr int kCStage = 32 * 2 * kCCols;
  static constexpr int oC = kTmaStore ? cround(oTs + ST * kTScaleSlot, 1024) : oTs + ST * kTScaleSlot;
  static constexpr int oCtl = oC + (kTmaStore ? 4 * 2 * kCStage : 0);
  static constexpr int kCtlBytes = 1024;
  static constexpr int kSmemBytes = oCtl + kCtlBytes + 1024;  // + alignment slack
  // tensor memory: accumulator (256 columns) | per B slot the A operand (token m at lane m,
  // 32 columns = 128 K codes) | per B slot 12 scale columns: 4 token (A) columns (lane m reads
  // column m / 32) then 8 weight (B) columns (row n at lane n % 32 of every lane quarter,
  // column n / 32). Lanes >= BM of the A slot are never written; they only reach accumulator
  // lanes >= BM, which are never stored.
  static constexpr int kACol0 = 256;
  static constexpr int kSfCols = 12;
  static constexpr int kSfCol0 = kACol0 + 32 * SB;
  static constexpr int kTmemCols = 512;
  static constexpr int kTranscodeWarps = 16;
  static constexpr int kGroupWarps = kTranscodeWarps / kGroups;
  static_assert(kGroupWarps == 4 || kGroupWarps == 8, "delivery roles need four or eight warps");
  static constexpr int kRowsPerThread = kBRows / (32 * kGroupWarps);
  static constexpr int kEpiWarps = 4;
  static constexpr int kTProducerWarp = 2 + kEpiWarps + kTranscodeWarps;  // 22
  static constexpr int kThreads = 32 * (kTProducerWarp + 1);
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kSfCol0 + SB * kSfCols <= kTmemCols, "tensor memory budget");
  static_assert(kSfCols % 4 == 0 && kSfCol0 % 4 == 0, "scale-factor addresses 4-column aligned");
  static_assert(oW % 1024 == 0 && oB % 1024 == 0 && kTRowBytes % 1024 == 0 &&
                    kWStage % 1024 == 0 && kBStage % 1024 == 0,
                "1 KB swizzle atoms");
  static_assert(kRowsPerThread >= 1, "a weight row per thread at least");
  static_assert(!kPair || kRowsPerThread == 1, "pairs: one weight row per thread");
  static_assert(oTs % 128 == 0 && kTScaleSlot % 128 == 0 && kWCodes % 128 == 0,
                "TMA shared-memory destinations 128-byte aligned");
  static_assert(!kTmaStore || (oC % 1024 == 0 && kCStage % 1024 == 0),
                "swizzled staging buffers 1 KB aligned");
  static_assert(SW <= 4 && SB <= 4 && ST <= 8, "control block sizes");
  static_assert(SW % kGroups == 0 && SB % kGroups == 0, "slots owned by one group");
  static_assert(!kGroupDelivers || ST % kGroups == 0, "token slots owned by one group");
  static_assert(8 * kPermCopies == (1 << kRowShift), "class-word shifts match the row stride");
};

struct GemmCtl {
  uint64_t wfull[4], wempty[4], tfull[8], tempty[8], bready[4], bempty[4], sfready[4];
  uint64_t acc_full, acc_empty, drain, fin_bar;
  uint32_t tmem_base;
  uint32_t fin_job;  // 1: this CTA finishes the tile of its last segment
  uint32_t abort_flag;
  uint32_t bcast;
  uint32_t sink;  // target of the never-taken dependent store of an early weight-stage release
  TranscodeTables tab;  // scale-byte classes (E4M3 sideband only)
};

struct GemmParams {
  void* out;                    // C, or the fp32 workspace planes (kOutPartial)
  float* slots;                 // stream-K partial slots [grid][2][BM][256]
  uint32_t* counters;           // stream-K per-tile arrival counters (zero between calls)
  const __nv_bfloat16* bias;
  float tensor_scale;
  int M, N, K;
  int n_tiles, m_tiles, nks;    // nks: 128-wide K chunks per tile
  int n_half_tiles;             // N / 128 (128-row halves of the packed weights)
  int split_k;                  // 0 = stream-K, else explicit split
  int split_out;                // output mode of explicit split segments
  int out_dtype, epilogue;
  int vec_out;                  // 1: C is 16-byte aligned (vector stores)
  int weights_early;            // 1: B is not written by the grid this one may overlap
  int fixup_kernel;             // 1: stream-K partials are summed by streamk_fixup_kernel
  int tma_c;                    // 1: whole 128-row tiles store C (16-bit) with TMA (tm_c)
  uint32_t* err;
};

// One contiguous run of chunks of one tile.
struct Seg {
  int tile, k0, k1, z, slot;  // slot: -1 full tile, 0/1 stream-K partial slot
};

// The work of CTA `c` of `G`: segment number `idx` (false when there is none). All indices
// fit 32 bits (the host rejects larger problems).
struct Schedule {
  int U;        // units (tile, chunk)
  int q, r;     // stream-K: U = q*G + r
  int G, nks, tiles, split;

  __device__ __forceinline__ void init(const GemmParams& p, int grid) {
    G = grid;
    nks = p.nks;
    tiles = p.n_tiles * p.m_tiles;
    split = p.split_k;
    U = tiles * nks;
    q = U / G;
    r = U % G;
  }
  __device__ __forceinline__ int u0(int c) const { return c * q + min(c, r); }
  __device__ __forceinline__ int cta_of(int u) const {
    const int big = r * (q + 1);
    return u < big ? u / (q + 1) : r + (u - big) / q;
  }
  __device__ __forceinline__ bool segment(int c, int idx, Seg& s) const {
    if (split > 0) {
      const int item = c + idx * G;
      if (item >= tiles * split) return false;
      s.tile = item / split;
      s.z = item % split;
      const int per = nks / split;
      s.k0 = s.z * per;
      s.k1 = s.k0 + per;
      s.slot = -1;
      return true;
    }
    const int a = u0(c), b = u0(c + 1);
    if (a >= b) return false;
    const int t = a / nks + idx;
    const int lo = max(a, t * nks), hi = min(b, (t + 1) * nks);
    if (lo >= hi) return false;
    s.tile = t;
    s.k0 = lo - t * nks;
    s.k1 = hi - t * nks;
    s.z = 0;
    s.slot = (s.k0 == 0 && s.k1 == nks) ? -1 : (idx == 0 ? 0 : 1);
    return true;
  }
};

// SiLU and tanh-GELU with every multiply and add rounded on its own (no contraction into FMAs,
// which the compiler may do differently in different drain loops): every store path of the
// GEMM gives the same bits.
__device__ __forceinline__ float silu_rn(float v) {
  return __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
}
__device__ __forceinline__ float gelu_tanh_rn(float v) {
  const float v3 = __fmul_rn(__fmul_rn(v, v), v);
  const float y = __fmul_rn(0.7978845608028654f, __fadd_rn(v, __fmul_rn(0.044715f, v3)));
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanhf(y)));
}

__device__ __forceinline__ float apply_epilogue(float v, int epi, const __nv_bfloat16* bias,
                                                int n) {
  if (epi != 0) v = __fadd_rn(v, __bfloat162float(bias[n]));
  if (epi == 2) v = fmaxf(v, 0.0f);
  else if (epi == 3) v = silu_rn(v);
  else if (epi == 4) v = gelu_tanh_rn(v);
  return v;
}

// The same for NV consecutive outputs n .. n + NV - 1, scaled first: the epilogue kind is
// tested once per row piece, not per element (a per-element test in an unrolled drain loop
// cost more than the conversion itself), with the same operations in the same order.
template <int NV>
__device__ __forceinline__ void apply_epilogue_row(float (&v)[NV], float scale, int epi,
                                                   const __nv_bfloat16* bias, int n) {
#pragma unroll
  for (int j = 0; j < NV; ++j) v[j] = __fmul_rn(v[j], scale);
  if (epi == 0) return;
#pragma unroll
  for (int j = 0; j < NV; ++j) v[j] = __fadd_rn(v[j], __bfloat162float(bias[n + j]));
  if (epi == 2) {
#pragma unroll
    for (int j = 0; j < NV; ++j) v[j] = fmaxf(v[j], 0.0f);
  } else if (epi == 3) {
#pragma unroll
    for (int j = 0; j < NV; ++j) v[j] = silu_rn(v[j]);
  } else if (epi == 4) {
#pragma unroll
    for (int j = 0; j < NV; ++j) v[j] = gelu_tanh_rn(v[j]);
  }
}

__device__ __forceinline__ void store_out(void* out, int64_t idx, float v, int dtype) {
  if (dtype == 0) reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  else if (dtype == 1) reinterpret_cast<__half*>(out)[idx] = __float2half_rn(v);
  else reinterpret_cast<float*>(out)[idx] = v;
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}


// NV consecutive outputs (element index idx, a multiple of NV) in the output dtype; vector
// stores (16 bytes, 8 for four 16-bit values) when C is 16-byte aligned.
template <int NV>
__device__ __forceinline__ void store_row(void* out, int64_t idx, const float (&v)[NV], int dtype,
                                          int vec) {
  if (!vec) {
#pragma unroll
    for (int j = 0; j < NV; ++j) store_out(out, idx + j, v[j], dtype);
    return;
  }
  if (dtype == 2) {
    float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + idx);
#pragma unroll
    for (int j = 0; j < NV / 4; ++j)
      o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    return;
  }
  uint32_t w[NV / 2];
#pragma unroll
  for (int j = 0; j < NV / 2; ++j) {
    if (dtype == 0) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&b);
    } else {
      const __half2 b = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&b);
    }
  }
  if constexpr (NV % 8 == 0) {
    uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + idx);
#pragma unroll
    for (int j = 0; j < NV / 8; ++j)
      o[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  } else {
    static_assert(NV == 4, "4, 8, 16 or 32 outputs");
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(out) + idx) = make_uint2(w[0], w[1]);
  }
}

// Eight E2M1 codes of a transcode-ready word (magnitudes in nibble bits 0..2; the signs of
// elements 0..3 at bits 7, 15, 23, 31 and of elements 4..7 at bits 3, 11, 19, 27) -> eight E4M3
// bytes, with the magnitude table T of the 16-block's class: one prmt per four magnitudes, the
// signs merged in place.
__device__ __forceinline__ void nib8_to_e4m3(uint32_t w, uint2 T, uint32_t& lo, uint32_t& hi) {
  const uint32_t m = w & 0x77777777u;
  lo = prmt(T.x, T.y, m) | (w & 0x80808080u);
  hi = prmt(T.x, T.y, m >> 16) | ((w << 4) & 0x80808080u);
}

// The same for a word of E2M1 codes as the reference stores them (sign in bit 3 of each
// nibble): byte i of (w<<4) / w carries the sign of element 2i / 2i+1 in bit 7, so one prmt
// gathers four of them.
__device__ __forceinline__ void nib8_natural_to_e4m3(uint32_t w, uint2 T, uint32_t& lo,
                                                     uint32_t& hi) {
  const uint32_t m = w & 0x77777777u;
  const uint32_t t = w << 4;
  lo = (prmt(t, w, 0x5140u) & 0x80808080u) | prmt(T.x, T.y, m);
  hi = (prmt(t, w, 0x7362u) & 0x80808080u) | prmt(T.x, T.y, m >> 16);
}

// Table rows (d*8 + mb) of the two 16-blocks of a 32-block and its E8M0 byte, from the two
// E4M3 scale bytes (the E4M3 sideband): the classes (e + 16) << 3 | mb come from the table,
// d = min(emax - e, 7), E8M0 = emax + 111.
__device__ __forceinline__ void pair_class(const TranscodeTables& t, uint32_t s0, uint32_t s1,
                                           uint32_t& i0, uint32_t& i1, uint32_t& e8) {
  const uint32_t c0 = t.info[s0 & 0x7Fu], c1 = t.info[s1 & 0x7Fu];
  const int e0 = static_cast<int>(c0 >> 3), e1 = static_cast<int>(c1 >> 3);
  const int em = max(e0, e1);
  i0 = static_cast<uint32_t>(min(em - e0, 7)) * 8u + (c0 & 7u);
  i1 = static_cast<uint32_t>(min(em - e1, 7)) * 8u + (c1 & 7u);
  e8 = static_cast<uint32_t>(em + 111);
}

// Stream-K fix-up of one tile: C = sum of the contributors' fp32 partial slots, added in CTA
// order (first..last), times the tensor scale, bias and activation. Worker `worker` of
// `nworkers` takes float4 groups worker, worker + nworkers, ...; loads of up to four
// contributors x two groups are in flight at once.
template <int BM>
__device__ __forceinline__ void streamk_reduce(const GemmParams& p, const Schedule& sch,
                                               const Seg& sg, int first, int last, int worker,
                                               int nworkers) {
  const int mt = sg.tile / p.n_tiles, nt = sg.tile % p.n_tiles;
  const int m0 = mt * BM, n0 = nt * kTileN;
  const int mrows = min(BM, p.M - m0);
  const int g4 = min(kTileN, p.N - n0) / 4;  // float4 groups per row
  const int total = mrows * g4;
  for (int g = worker; g < total; g += 2 * nworkers) {
    float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    int off[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int gi = g + u * nworkers;
      const int rr = gi / g4;
      off[u] = rr * kTileN + (gi - rr * g4) * 4;
    }
    for (int c = first; c <= last; c += 4) {
      float4 v[4][2];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int ci = c + cc;
        const int sl = (sch.u0(ci) / p.nks == sg.tile) ? 0 : 1;
        const float* base = p.slots + (static_cast<int64_t>(ci) * 2 + sl) * (BM * kTileN);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          v[cc][u] = (ci <= last && g + u * nworkers < total)
                         ? __ldcg(reinterpret_cast<const float4*>(base + off[u]))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          acc[u].x += v[cc][u].x;
          acc[u].y += v[cc][u].y;
          acc[u].z += v[cc][u].z;
          acc[u].w += v[cc][u].w;
        }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int gi = g + u * nworkers;
      if (gi >= total) break;
      const int rr = off[u] / kTileN, n = n0 + (off[u] - rr * kTileN);
      float o[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
      apply_epilogue_row<4>(o, p.tensor_scale, p.epilogue, p.bias, n);
      store_row<4>(p.out, static_cast<int64_t>(m0 + rr) * p.N + n, o, p.out_dtype, p.vec_out);
    }
  }
}

// Number of segments of CTA c and whether the last one is a stream-K partial.
__device__ __forceinline__ int last_segment(const Schedule& sch, int c, Seg& last) {
  int n = 0;
  Seg sg;
  while (sch.segment(c, n, sg)) {
    last = sg;
    ++n;
  }
  return n;
}

// 16 or 32 consecutive accumulator columns of this warp's lane quarter into registers.
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
  static_assert(N == 16 || N == 32, "16 or 32 columns");
  if constexpr (N == 16) tmem_ld_x16(taddr, r);
  else tmem_ld_x32(taddr, r);
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Token row `mrow` of token slot `ts` (one E2M3 code per byte, 128B-swizzled as the TMA wrote
// it) into the tensor-memory A slot at `dst` (this warp's lane quarter, lane = token row);
// rows >= BM are written as zeros. The bytes go over as they are: the MMA reads an E2M3
// element of tensor memory from bits 0..5 of its byte and ignores bits 6..7 (the in-place
// activation test sets them), so clearing them (32 ALU instructions per row and chunk, 2-5 %
// of the prefill GEMM) is not needed. Returns a word that depends on one word of every load (a
// vector load's words complete together), for release_after_loads. Executed by a whole warp.
template <class Cfg>
__device__ __forceinline__ uint32_t copy_token_rows(const uint8_t* smem, int ts, int mrow,
                                                    uint32_t dst) {
  uint32_t av[32];
  uint32_t dep = 0u;
  if (mrow < Cfg::kRows) {
    const uint8_t* trow =
        smem + Cfg::oT + ts * Cfg::kTRowBytes + (mrow >> 3) * 1024 + (mrow & 7) * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(trow + ((c ^ (mrow & 7)) << 4));
      av[4 * c + 0] = v.x;
      av[4 * c + 1] = v.y;
      av[4 * c + 2] = v.z;
      av[4 * c + 3] = v.w;
      dep ^= v.x;
    }
  } else {
#pragma unroll
    for (int c = 0; c < 32; ++c) av[c] = 0u;
  }
  tmem_st_x32(dst, av);
  return dep;
}

// Arrive on `bar` once every shared-memory load whose value `dep` depends on has completed:
// an empty asm that takes `dep` orders nothing at run time, and an asynchronous consumer of
// the loaded registers (tcgen05.st) need not hold the warp, so a comparison on `dep` (its store
// is never taken) makes the warp wait for those loads before the arrive. A slot refilled by TMA
// while a load of it was still in flight would hand that load the next chunk's data.
__device__ __forceinline__ void release_after_loads(uint32_t dep, int lane, uint32_t bar,
                                                    volatile uint32_t* sink) {
  if (dep == 0x9E3779B9u && lane == 31) *sink = dep;
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// kClassWords: B in bd_pack_b's transcode-ready layout (moved sign bits, class words); else
// the E4M3 sideband (bd_pack_b_e4m3: the reference's codes and scale bytes, regrouped).
template <int BM, bool kClassWords>
__global__ void __launch_bounds__(GemmCfg<BM>::kThreads, 1)
    w4a6_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_as,
                     const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_ws,
                     const __grid_constant__ CUtensorMap tm_c, const GemmParams p) {
  using Cfg = GemmCfg<BM>;
  static_assert(sizeof(GemmCtl) <= Cfg::kCtlBytes, "control block");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  GemmCtl& ctl = *reinterpret_cast<GemmCtl*>(smem + Cfg::oCtl);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // CTA pairs: the schedule deals tiles to clusters; `rank` picks this CTA's token and weight
  // rows of the tile
  const uint32_t rank = Cfg::kPair ? cluster_ctarank() : 0u;
  const int cta = Cfg::kPair ? static_cast<int>(blockIdx.x / 2) : static_cast<int>(blockIdx.x);
  volatile uint32_t* abort_flag = &ctl.abort_flag;
  Schedule sch;
  sch.init(p, Cfg::kPair ? gridDim.x / 2 : gridDim.x);
  // pair barriers the peer CTA arrives on, as shared::cluster addresses in rank 0 (bready,
  // acc_empty) and in the peer (sfready)
  const uint32_t peer = rank ^ 1u;

  if (tid == 0) {
    ctl.abort_flag = 0;
    for (int s = 0; s < Cfg::SW; ++s) {
      mbar_init(smem_u32(&ctl.wfull[s]), 1);
      mbar_init(smem_u32(&ctl.wempty[s]), Cfg::kGroupWarps);
    }
    for (int s = 0; s < Cfg::ST; ++s) {
      mbar_init(smem_u32(&ctl.tfull[s]), 1);
      // released early by the four epilogue warps, or by the four warps of the group that
      // delivers the slot (pairs); else by the MMA's commit
      mbar_init(smem_u32(&ctl.tempty[s]), Cfg::kEarlyRelease ? 4 : 1);
    }
    // pairs: bready and acc_empty of rank 0 count both CTAs' epilogue warps, sfready of each
    // CTA both CTAs' transcode groups; the commits of the pair MMAs arrive once in each CTA
    constexpr int kPairs = Cfg::kPair ? 2 : 1;
    for (int s = 0; s < Cfg::SB; ++s) {
      mbar_init(smem_u32(&ctl.bready[s]),
                kPairs * (Cfg::kGroupDelivers ? Cfg::kGroupWarps : Cfg::kEpiWarps));
      mbar_init(smem_u32(&ctl.bempty[s]), 1);
      mbar_init(smem_u32(&ctl.sfready[s]), Cfg::kGroupWarps);
    }
    mbar_init(smem_u32(&ctl.acc_full), 1);
    mbar_init(smem_u32(&ctl.acc_empty), kPairs * Cfg::kEpiWarps);
    mbar_init(smem_u32(&ctl.drain), 1);
    mbar_init(smem_u32(&ctl.fin_bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  // the peer arrives on these barriers: both CTAs' are initialised before anyone arrives
  if constexpr (Cfg::kPair) cluster_sync_all();
  // a grid launched after this one with programmatic serialisation may be scheduled now; it
  // takes this SM only after this CTA exits, and waits for this grid before it reads A or
  // touches C and the workspace
  grid_dep_launch_dependents();
  // The producers start at once. Everything that needs tensor memory or the transcode tables
  // meets at named barrier 2 (warps 1..21) after warp 1 allocated and the transcode warps
  // copied the tables.
  uint32_t tbase = 0;
  if (warp >= 1 && warp < Cfg::kTProducerWarp) {
    if (warp == 1) {
      if constexpr (Cfg::kPair) {
        tmem_alloc_pair(smem_u32(&ctl.tmem_base), Cfg::kTmemCols);
        tmem_relinquish_pair();
      } else {
        tmem_alloc(smem_u32(&ctl.tmem_base), Cfg::kTmemCols);
        tmem_relinquish();
      }
    } else if (warp >= 2 + Cfg::kEpiWarps) {
      const int t0 = tid - 32 * (2 + Cfg::kEpiWarps);
      if constexpr (!kClassWords) load_tables<true>(ctl.tab, t0, 32 * Cfg::kTranscodeWarps);
      const uint2* src = reinterpret_cast<const uint2*>(&g_tables_e4m3);  // perm[] comes first
      uint2* rep = reinterpret_cast<uint2*>(smem + Cfg::oPerm);
      for (int i = t0; i < 64 * Cfg::kPermCopies; i += 32 * Cfg::kTranscodeWarps)
        rep[i] = __ldg(src + i / Cfg::kPermCopies);
    }
    tc_fence_before();
    named_barrier(2, 32 * (Cfg::kTProducerWarp - 1));
    tc_fence_after();
    tbase = ctl.tmem_base;
  }

  if (warp == 0) {
    // ------------------------------------------------------------------ weight producer
    if (lane == 0) {
      prefetch_tmap(&tm_w);
      prefetch_tmap(&tm_ws);
      if (!p.weights_early) grid_dep_wait();
      RingPos<Cfg::SW> w;
      Seg sg;
      for (int idx = 0; sch.segment(cta, idx, sg) && !*abort_flag; ++idx) {
        const int nt = sg.tile % p.n_tiles;
        // the second 128-row half is missing in the last tile when N / 128 is odd (pair tiles
        // need N % 256 == 0: each CTA loads its own half)
        const bool two = !Cfg::kPair && 2 * nt + 1 < p.n_half_tiles;
        const uint32_t tx = (two || Cfg::kPair) ? Cfg::kWStage : Cfg::kWStage / 2;
        // (half tile, chunk) row of the packed weights: the tile's first half; a CTA of a pair
        // loads the codes of its own half and the scales of both
        int row0 = (2 * nt) * p.nks + sg.k0;
        const int own = static_cast<int>(rank) * p.nks;
        for (int k = sg.k0; k < sg.k1; ++k, ++row0) {
          if (!mbar_wait(smem_u32(&ctl.wempty[w.slot]), w.phase ^ 1u, p.err, kErrWaitEmpty,
                         abort_flag))
            break;
          uint8_t* st = smem + Cfg::oW + w.slot * Cfg::kWStage;
          const uint32_t fb = smem_u32(&ctl.wfull[w.slot]);
          mbar_arrive_expect_tx(fb, tx);
          tma_load_2d(smem_u32(st), &tm_w, 0, (row0 + own) * 128, fb);
          tma_load_2d(smem_u32(st + Cfg::kWCodes), &tm_ws, 0, row0, fb);
          if (two || Cfg::kPair)
            tma_load_2d(smem_u32(st + Cfg::kWCodes + 1024), &tm_ws, 0, row0 + p.nks, fb);
          if (two) tma_load_2d(smem_u32(st + 8192), &tm_w, 0, (row0 + p.nks) * 128, fb);
          w.next();
        }
      }
    }
  } else if (warp == Cfg::kTProducerWarp) {
    // ------------------------------------------------------------------ token producer
    if (lane == 0) {
      prefetch_tmap(&tm_a);
      prefetch_tmap(&tm_as);
      grid_dep_wait();  // A may be written by the previous grid
      RingPos<Cfg::ST> t;
      Seg sg;
      for (int idx = 0; sch.segment(cta, idx, sg) && !*abort_flag; ++idx) {
        const int mt = sg.tile / p.n_tiles;
        for (int k = sg.k0; k < sg.k1; ++k) {
          if (!mbar_wait(smem_u32(&ctl.tempty[t.slot]), t.phase ^ 1u, p.err, kErrWaitEmpty,
                         abort_flag))
            break;
          uint8_t* st = smem + Cfg::oT + t.slot * Cfg::kTRowBytes;
          const uint32_t fb = smem_u32(&ctl.tfull[t.slot]);
          mbar_arrive_expect_tx(fb, Cfg::kTTx);
          const int m0 = mt * BM + static_cast<int>(rank) * Cfg::kRows;
          tma_load_3d(smem_u32(st), &tm_a, 0, m0, k, fb);
          tma_load_2d(smem_u32(smem + Cfg::oTs + t.slot * Cfg::kTScaleSlot), &tm_as, m0, k, fb);
          t.next();
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // (pairs: rank 0 issues for both CTAs, its commits arrive in both). The whole warp runs the
    // loop, its waits and addresses warp-uniform, and one elected lane issues the MMAs and
    // commits. Issued from lane 0 alone (a divergent single-thread loop) the same MMAs ran at
    // 240 cycles each instead of 128 whenever ALU-bound warps shared the warp's scheduler (a
    // probe of this loop: 968 against 512 cycles per chunk of four pair MMAs); warp-wide, 512
    // with or without them.
    if (rank == 0) {
      auto commit = [&](uint64_t& bar) {
        if constexpr (Cfg::kPair) tc_commit_pair(smem_u32(&bar), 3);
        else tc_commit(smem_u32(&bar));
      };
      RingPos<Cfg::SB> b;
      RingPos<Cfg::ST> t;
      Seg sg;
      for (int idx = 0; sch.segment(cta, idx, sg); ++idx) {
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&ctl.acc_empty), (idx & 1) ^ 1u, p.err,
                                               kErrWaitAccum, abort_flag)))
          break;
        tc_fence_after();
        bool ok = true;
        for (int k = sg.k0; k < sg.k1; ++k) {
          // bready: the B tile, its scales and the token operand (copied into tensor memory
          // after the token slot landed) are all in place (in both CTAs of a pair)
          if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&ctl.bready[b.slot]), b.phase, p.err,
                                                 kErrWaitOperand, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = smem_u32(smem + Cfg::oB + b.slot * Cfg::kBStage);
          const uint32_t ta = tbase + Cfg::kACol0 + b.slot * 32;
          const uint32_t sfa = tbase + Cfg::kSfCol0 + b.slot * Cfg::kSfCols;
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t acc = (k == sg.k0 && kk == 0) ? 0u : 1u;
              if constexpr (Cfg::kPair) {
                const uint32_t idesc = idesc_mxf8f6f4(256, kTileN, kFmtE2M3, kFmtE4M3, kk, kk);
                mma_mxf8f6f4_ts_pair(tbase, ta + kk * 8, sdesc_sw128(b_addr + kk * 32), idesc,
                                     sfa, sfa + 4, acc);
              } else {
                const uint32_t idesc = idesc_mxf8f6f4(128, kTileN, kFmtE2M3, kFmtE4M3, kk, kk);
                mma_mxf8f6f4_ts(tbase, ta + kk * 8, sdesc_sw128(b_addr + kk * 32), idesc, sfa,
                                sfa + 4, acc);
              }
            }
            commit(ctl.bempty[b.slot]);
            if constexpr (!Cfg::kEarlyRelease) commit(ctl.tempty[t.slot]);
          }
          __syncwarp();
          b.next();
          t.next();
        }
        if (elect_one()) commit(ctl.acc_full);
        __syncwarp();
        if (!ok) break;
      }
      // arrives once every tcgen05 operation this warp issued has completed
      if (elect_one()) commit(ctl.drain);
      __syncwarp();
    }
  } else if (warp >= 2 + Cfg::kEpiWarps) {
    // ------------------------------------------------------------------ transcode
    // The 16 warps form kGroups groups that take alternate chunks, so several chunks are in
    // flight at once; in a group, thread (warp gw, lane) converts all four K blocks of weight
    // row 32 gw + lane.
    const int tw = warp - 2 - Cfg::kEpiWarps;  // 0..15
    const int grp = tw / Cfg::kGroupWarps;
    constexpr int R = Cfg::kRowsPerThread;
    // rows of this thread: 32 (tw % group warps) + lane + 32 * group warps * r
    int code_sw[R], scale_off[R], b_sw[R], rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = r * (32 * Cfg::kGroupWarps) + (tw % Cfg::kGroupWarps) * 32 + lane;
      const int rr = row & 127;
      rows[r] = row;
      // raw codes: 64B-swizzled 128-row halves, 16-byte chunk c of row rr at
      // rr*64 + ((c ^ ((rr >> 1) & 3)) << 4); chunk c holds K block c
      // the row offset has zero bits 4..5 and the stage base is 1 KB aligned, so the address
      // of chunk c is (stage + row offset + swizzle << 4) ^ (c << 4)
      code_sw[r] = (row >> 7) * 8192 + rr * 64 + (((rr >> 1) & 3) << 4);
      scale_off[r] = Cfg::kWCodes + ((row >> 7) + static_cast<int>(rank)) * 1024 + rr * 8;
      // B operand: 128B-swizzled K-major, 16-byte chunk cc of row n at
      // (n >> 3)*1024 + (n & 7)*128 + ((cc ^ (n & 7)) << 4); block b covers chunks 2b, 2b + 1
      // likewise bits 4..6: chunk cc of row n at (slot + row offset + ((n & 7) << 4)) ^ (cc << 4)
      b_sw[r] = (row >> 3) * 1024 + (row & 7) * 128 + ((row & 7) << 4);
    }
    // The stage bases are 1 KB aligned and the swizzles touch address bits 4..6 only, so
    // (base + offset) ^ (c << 4) == base + (offset ^ (c << 4)): the swizzled offsets of this
    // thread's first row are computed once, a further row of the thread is a fixed distance
    // on (rows 128 apart), and every access is a warp-uniform base plus a per-thread offset.
    static_assert(R == 1 || 32 * Cfg::kGroupWarps == 128, "further rows 128 rows on");
    constexpr int kCodeRowStep = 8192, kScaleRowStep = 1024, kBRowStep = 16384;
    uint32_t code_off[4], b_off[8];
#pragma unroll
    for (int c = 0; c < 4; ++c) code_off[c] = static_cast<uint32_t>(code_sw[0]) ^ (c << 4);
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) b_off[cc] = static_cast<uint32_t>(b_sw[0]) ^ (cc << 4);
    // magnitude table: this lane's copy, as an offset OR-ed into each row's offset
    const uint8_t* tab_p = smem + Cfg::oPerm;
    const uint32_t lane_copy = (lane % Cfg::kPermCopies) * 8;
    int ci = 0;  // chunk number within this CTA
    Seg sg;
    for (int idx = 0; sch.segment(cta, idx, sg) && !*abort_flag; ++idx) {
      for (int k = sg.k0; k < sg.k1; ++k, ++ci) {
        if (ci % Cfg::kGroups != grp) continue;
        const int ws = ci % Cfg::SW, bs = ci % Cfg::SB;
        const uint32_t wph = (ci / Cfg::SW) & 1, bph = (ci / Cfg::SB) & 1;
        if (!mbar_wait(smem_u32(&ctl.wfull[ws]), wph, p.err, kErrWaitTma, abort_flag)) break;
        const uint8_t* st = smem + Cfg::oW + ws * Cfg::kWStage;
        uint4 q[R][4];
        uint2 sc[R];
        const uint32_t st_u = smem_u32(st);
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
          for (int c = 0; c < 4; ++c) q[r][c] = ld_shared_v4(st_u + code_off[c] + r * kCodeRowStep);
          sc[r] = *reinterpret_cast<const uint2*>(st + scale_off[0] + r * kScaleRowStep);
        }
        // pairs: the peer half's class words of this thread's row (for its E8M0 word), loaded
        // with the rest before the stage is released
        uint2 sp = make_uint2(0u, 0u);
        if constexpr (Cfg::kPair)
          sp = *reinterpret_cast<const uint2*>(st + Cfg::kWCodes + static_cast<int>(peer) * 1024 +
                                               rows[0] * 8);
        if constexpr (Cfg::kEarlyRelease) {
          // Release the weight stage now: a store that depends on every load (never taken, but
          // the loads must complete before it can issue; one word of a vector load completes
          // with the others) comes before the arrive, so no load of the stage is pending when
          // its next TMA fill lands.
          uint32_t dep = sp.x;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            dep ^= sc[r].x;
#pragma unroll
            for (int c = 0; c < 4; ++c) dep ^= q[r][c].x;
          }
          release_after_loads(dep, lane, smem_u32(&ctl.wempty[ws]),
                              reinterpret_cast<volatile uint32_t*>(&ctl.sink));
        }
        // Otherwise the weight stage is released only after the B rows computed from it are stored
        // (below), never straight after the loads: the stores depend on every loaded word, so
        // the stage cannot be refilled while a load of it is still outstanding. An arrive
        // right after the loads (a release that orders this thread's stores, not its loads)
        // let the next fill of the stage land before some loads were performed when the
        // bempty wait stalled (segment boundaries of long stream-K schedules): those rows came
        // out converted from the chunk four places later. Volatile loads did not prevent it;
        // folding every loaded word into a value stored before the arrive did, at no gain.
        if (!mbar_wait(smem_u32(&ctl.bempty[bs]), bph ^ 1u, p.err, kErrWaitMma, abort_flag))
          break;
        const uint32_t bt = smem_u32(smem + Cfg::oB + bs * Cfg::kBStage);
        uint32_t* sf_stage = reinterpret_cast<uint32_t*>(smem + Cfg::oSf + bs * 1024);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          uint32_t sfw = 0;
#pragma unroll
          for (int blk = 0; blk < 4; ++blk) {
            const uint32_t f = blk < 2 ? (sc[r].x >> (16 * blk)) : (sc[r].y >> (16 * (blk - 2)));
            uint32_t off0, off1;  // byte offsets of the two 16-blocks' table rows
            if constexpr (kClassWords) {
              // class word: both rows times the table's row stride (bits 0..5: the smaller
              // exponent's row, bits 6..8: the other's mantissa bits = its row)
              constexpr int kS = Cfg::kRowShift;
              const uint32_t off_small = ((f << kS) & (0x3Fu << kS)) | lane_copy;
              const uint32_t off_big = ((f << (kS - 6)) & (0x7u << kS)) | lane_copy;
              const bool first_big = (f & 0x200u) != 0;
              off0 = first_big ? off_big : off_small;
              off1 = first_big ? off_small : off_big;
            } else {
              uint32_t i0, i1, e8;
              pair_class(ctl.tab, f & 0xFFu, (f >> 8) & 0xFFu, i0, i1, e8);
              off0 = (i0 * (8 * Cfg::kPermCopies)) | lane_copy;
              off1 = (i1 * (8 * Cfg::kPermCopies)) | lane_copy;
              sfw |= e8 << (8 * blk);
            }
            const uint2 T0 = *reinterpret_cast<const uint2*>(tab_p + off0);
            const uint2 T1 = *reinterpret_cast<const uint2*>(tab_p + off1);
            uint32_t v[8];
            if constexpr (kClassWords) {
              nib8_to_e4m3(q[r][blk].x, T0, v[0], v[1]);
              nib8_to_e4m3(q[r][blk].y, T0, v[2], v[3]);
              nib8_to_e4m3(q[r][blk].z, T1, v[4], v[5]);
              nib8_to_e4m3(q[r][blk].w, T1, v[6], v[7]);
            } else {
              nib8_natural_to_e4m3(q[r][blk].x, T0, v[0], v[1]);
              nib8_natural_to_e4m3(q[r][blk].y, T0, v[2], v[3]);
              nib8_natural_to_e4m3(q[r][blk].z, T1, v[4], v[5]);
              nib8_natural_to_e4m3(q[r][blk].w, T1, v[6], v[7]);
            }
            st_shared_v4(bt + b_off[2 * blk] + r * kBRowStep, v[0], v[1], v[2], v[3]);
            st_shared_v4(bt + b_off[2 * blk + 1] + r * kBRowStep, v[4], v[5], v[6], v[7]);
          }
          // E8M0 bytes of the row's four 32-blocks (class words: bits 10..14 + 118)
          if constexpr (kClassWords)
            sfw = prmt((sc[r].x >> 10) & 0x001F001Fu, (sc[r].y >> 10) & 0x001F001Fu, 0x6420u) +
                  0x76767676u;
          sf_stage[static_cast<int>(rank) * Cfg::kBRows + rows[r]] = sfw;
          if constexpr (Cfg::kPair) {
            // each CTA's MMA reads the scales of all 256 weight rows from its own tensor memory:
            // the E8M0 words of the peer half's row too (R == 1 in pairs)
            uint32_t sfp = 0;
            if constexpr (kClassWords) {
              sfp = prmt((sp.x >> 10) & 0x001F001Fu, (sp.y >> 10) & 0x001F001Fu, 0x6420u) +
                    0x76767676u;
            } else {
#pragma unroll
              for (int blk = 0; blk < 4; ++blk) {
                const uint32_t f = blk < 2 ? (sp.x >> (16 * blk)) : (sp.y >> (16 * (blk - 2)));
                uint32_t i0, i1, e8;
                pair_class(ctl.tab, f & 0xFFu, (f >> 8) & 0xFFu, i0, i1, e8);
                sfp |= e8 << (8 * blk);
              }
            }
            sf_stage[static_cast<int>(peer) * Cfg::kBRows + rows[r]] = sfp;
          }
        }
        fence_proxy_async_smem();  // the tensor core reads the B tile through the async proxy
        __syncwarp();
        if (lane == 0) {
          if constexpr (!Cfg::kEarlyRelease) mbar_arrive(smem_u32(&ctl.wempty[ws]));
          mbar_arrive(smem_u32(&ctl.sfready[bs]));
        }
        if constexpr (Cfg::kGroupDelivers) {
          // The chunk's operands into tensor memory, by this group: warps 0..3 of the group (one
          // per lane quarter) the quarter's token rows and token scales; the weight scales, once
          // every warp of the group has staged its rows' words (sfready; a bounded wait, so a
          // warp that gave up earlier makes this one time out, not hang), by warps 4..7 of an
          // eight-warp group and by every warp of a four-warp group. The MMA waits for all the
          // group's warps (bready).
          const int quarter = warp & 3;
          const int mrow = quarter * 32 + lane;
          const uint32_t taddr = tbase + (static_cast<uint32_t>(quarter * 32) << 16);
          const uint32_t col = taddr + Cfg::kSfCol0 + bs * Cfg::kSfCols;
          const int ts = ci % Cfg::ST;
          const int gw = tw % Cfg::kGroupWarps;
          const bool sf_role = Cfg::kGroupWarps == 4 || gw >= 4;
          bool ok = true;
          if (gw < 4) {
            ok = mbar_wait(smem_u32(&ctl.tfull[ts]), (ci / Cfg::ST) & 1, p.err, kErrWaitTma,
                           abort_flag);
            if (ok) {
              uint32_t dep = 0u;
              if (quarter * 32 < Cfg::kRows)
                dep = copy_token_rows<Cfg>(smem, ts, mrow, taddr + Cfg::kACol0 + bs * 32);
              const uint32_t* tok =
                  reinterpret_cast<const uint32_t*>(smem + Cfg::oTs + ts * Cfg::kTScaleSlot);
              const uint32_t tokw = mrow < Cfg::kRows ? tok[mrow] : 0u;
              // the token rows and the scale are in registers: the token slot can be refilled
              // (the four warps of the group)
              if constexpr (Cfg::kEarlyRelease)
                release_after_loads(dep ^ tokw, lane, smem_u32(&ctl.tempty[ts]),
                                    reinterpret_cast<volatile uint32_t*>(&ctl.sink));
              tmem_st_x1(col + quarter, tokw);
            }
          }
          if (ok && sf_role) {
            ok = mbar_wait(smem_u32(&ctl.sfready[bs]), (ci / Cfg::SB) & 1, p.err,
                           kErrWaitOperand, abort_flag);
            if (ok) {
              uint32_t wv[8];
#pragma unroll
              for (int c = 0; c < 8; ++c) wv[c] = sf_stage[32 * c + lane];
              tmem_st_x8(col + 4, wv);
            }
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (!ok) break;
          if (lane == 0) {
            if (Cfg::kPair && rank != 0) mbar_arrive_remote(mapa_shared(smem_u32(&ctl.bready[bs]), 0));
            else mbar_arrive(smem_u32(&ctl.bready[bs]));
          }
        }
      }
    }
    // the fix-up of the tile of this CTA's last segment, when this CTA finishes it, is shared
    // with the epilogue warps (workers 128.. of 640)
    Seg lastseg;
    if (p.split_k == 0 && !p.fixup_kernel && last_segment(sch, cta, lastseg) > 0 &&
        lastseg.slot >= 0 &&
        !*abort_flag &&
        mbar_wait(smem_u32(&ctl.fin_bar), 0, p.err, kErrWaitAccum, abort_flag) &&
        ctl.fin_job != 0) {
      const int first = sch.cta_of(lastseg.tile * p.nks);
      const int last = sch.cta_of((lastseg.tile + 1) * p.nks - 1);
      streamk_reduce<BM>(p, sch, lastseg, first, last, 32 * Cfg::kEpiWarps + 32 * tw + lane,
                         32 * (Cfg::kEpiWarps + Cfg::kTranscodeWarps));
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;
    const int ep_tid = tid - 64;  // 0..127
    const int mrow = quarter * 32 + lane;  // token row of the tile (accumulator lane)
    // accumulator columns per tensor-memory load: 32 for decode tiles (half the load round trips
    // of a drain), 16 for 128-row tiles (measured faster there)
    constexpr int kEB = BM <= 64 ? 32 : 16;
    grid_dep_wait();  // C, bias and the workspace belong to the previous grid until it ends
    const uint32_t taddr = tbase + (static_cast<uint32_t>(quarter * 32) << 16);
    Seg lastseg;
    const int nseg = last_segment(sch, cta, lastseg);
    // this warp's C staging buffers and the count of its TMA stores (kTmaStore)
    const uint32_t cstage = smem_u32(smem + Cfg::oC) + quarter * 2 * Cfg::kCStage;
    int c_stores = 0;
    RingPos<Cfg::SB> b;
    RingPos<Cfg::ST> t;
    Seg sg;
    for (int idx = 0; sch.segment(cta, idx, sg) && !*abort_flag; ++idx) {
      // Scale factors of each chunk of this segment into tensor memory, in this warp's lane
      // quarter: token m = 32 quarter + lane at column quarter, weight row 32c + lane at
      // column 4 + c (every quarter holds a copy of the weight scales). Staged by the
      // transcode warps (sfready); the MMA waits for all four quarters (bready).
      bool ok = true;
      for (int k = sg.k0; k < sg.k1 && !Cfg::kGroupDelivers; ++k) {
        if (!mbar_wait(smem_u32(&ctl.sfready[b.slot]), b.phase, p.err, kErrWaitOperand,
                       abort_flag) ||
            !mbar_wait(smem_u32(&ctl.tfull[t.slot]), t.phase, p.err, kErrWaitTma, abort_flag)) {
          ok = false;
          break;
        }
        uint32_t dep = 0u;
        if (quarter * 32 < Cfg::kRows)
          dep = copy_token_rows<Cfg>(smem, t.slot, mrow, taddr + Cfg::kACol0 + b.slot * 32);
        const uint32_t* tok = reinterpret_cast<const uint32_t*>(
            smem + Cfg::oTs + t.slot * Cfg::kTScaleSlot);
        const uint32_t tokw = mrow < Cfg::kRows ? tok[mrow] : 0u;
        // the token rows and the scale are in registers: the token slot can be refilled
        if constexpr (Cfg::kEarlyRelease)
          release_after_loads(dep ^ tokw, lane, smem_u32(&ctl.tempty[t.slot]),
                              reinterpret_cast<volatile uint32_t*>(&ctl.sink));
        const uint32_t* sf_stage = reinterpret_cast<const uint32_t*>(smem + Cfg::oSf + b.slot * 1024);
        uint32_t wv[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) wv[c] = sf_stage[32 * c + lane];
        const uint32_t col = taddr + Cfg::kSfCol0 + b.slot * Cfg::kSfCols;
        tmem_st_x1(col + quarter, tokw);
        tmem_st_x8(col + 4, wv);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (Cfg::kPair && rank != 0) mbar_arrive_remote(mapa_shared(smem_u32(&ctl.bready[b.slot]), 0));
          else mbar_arrive(smem_u32(&ctl.bready[b.slot]));
        }
        b.next();
        t.next();
      }
      if (!ok) break;
      if (!mbar_wait(smem_u32(&ctl.acc_full), idx & 1, p.err, kErrWaitAccum, abort_flag))
        break;
      tc_fence_after();
      const int mt = sg.tile / p.n_tiles, nt = sg.tile % p.n_tiles;
      // this CTA's token rows of the tile (pairs: rank r holds rows 128 r ..)
      const int m0 = mt * BM + static_cast<int>(rank) * Cfg::kRows, n0 = nt * kTileN;
      const int mrows = min(Cfg::kRows, p.M - m0);  // valid token rows (may be <= 0 in a pair)
      const int ncols = min(kTileN, p.N - n0);      // valid weight rows (multiple of 128)
      const bool warp_rows = quarter * 32 < mrows;
      const bool row_ok = mrow < mrows;
      const int m = m0 + mrow;
      if (sg.slot >= 0) {
        // stream-K partial: store it in this CTA's slot, free the accumulator, count the
        // arrivals for this tile; the last contributor sums all slots in CTA order (so the
        // result does not depend on which CTA arrived last), all 128 threads sharing the work
        float* slot = p.slots + (static_cast<int64_t>(cta) * 2 + sg.slot) * (BM * kTileN);
        if (warp_rows) {
          for (int c0 = 0; c0 < ncols; c0 += kEB) {
            uint32_t r[kEB];
            __syncwarp();
            tmem_ld_cols<kEB>(taddr + c0, r);
            tmem_ld_wait();
            if (row_ok) {
              float4* dst = reinterpret_cast<float4*>(slot + mrow * kTileN + c0);
#pragma unroll
              for (int j = 0; j < kEB / 4; ++j)
                __stcg(dst + j, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                            __uint_as_float(r[4 * j + 2]),
                                            __uint_as_float(r[4 * j + 3])));
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (Cfg::kPair && rank != 0) mbar_arrive_remote(mapa_shared(smem_u32(&ctl.acc_empty), 0));
          else mbar_arrive(smem_u32(&ctl.acc_empty));
        }
        if (p.fixup_kernel) continue;  // summed after this grid by streamk_fixup_kernel
        const int first = sch.cta_of(sg.tile * p.nks);
        const int last = sch.cta_of((sg.tile + 1) * p.nks - 1);
        // the count-in (acquire-release at GPU scope, after the barrier that follows every
        // epilogue thread's partial stores) publishes this CTA's partial and, for the last
        // contributor, makes the others' visible; the barriers below and the fin_bar
        // handshake carry that to the threads that sum (no separate fences: each cost the
        // decode GEMM 2-4 %)
        named_barrier(1, 32 * Cfg::kEpiWarps);
        if (ep_tid == 0) {
          const uint32_t old = atom_add_acq_rel_gpu(p.counters + sg.tile, 1u);
          const bool fin = old == static_cast<uint32_t>(last - first);
          if (fin) p.counters[sg.tile] = 0;  // every contributor has arrived: rearm
          ctl.bcast = fin ? 1u : 0u;
        }
        named_barrier(1, 32 * Cfg::kEpiWarps);
        const bool finish = ctl.bcast != 0;
        named_barrier(1, 32 * Cfg::kEpiWarps);
        const bool helped = idx == nseg - 1;  // the transcode warps are idle by then
        if (helped && ep_tid == 0) {
          ctl.fin_job = finish ? 1u : 0u;
          mbar_arrive(smem_u32(&ctl.fin_bar));
        }
        if (finish) {
          streamk_reduce<BM>(p, sch, sg, first, last, ep_tid,
                             helped ? 32 * (Cfg::kEpiWarps + Cfg::kTranscodeWarps)
                                    : 32 * Cfg::kEpiWarps);
        }
        continue;
      }
      if constexpr (Cfg::kTmaStore) {
        if (p.tma_c) {
          // kCCols columns per TMA store, loaded 32 at a time, converted to 16-bit, staged
          // (row = lane, swizzled as the store's map) and stored by one TMA store per warp,
          // which clips rows >= M; a staging buffer is rewritten once the store issued two
          // steps earlier has read it. (Loading the next 32 columns while staging this piece
          // needed more than the 80 registers a thread has here: the spills made it 5 %
          // slower; so did 16-column loads with the next piece in flight.)
          // The accumulator is released as soon as its last columns are in registers, before
          // they are converted and stored.
          auto release_acc = [&]() {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
              if (Cfg::kPair && rank != 0) mbar_arrive_remote(mapa_shared(smem_u32(&ctl.acc_empty), 0));
              else mbar_arrive(smem_u32(&ctl.acc_empty));
            }
          };
          if (warp_rows) {
            for (int c0 = 0; c0 < ncols; c0 += Cfg::kCCols) {
              const uint32_t sb = cstage + (c_stores & 1) * Cfg::kCStage;
              if (c_stores >= 2) {
                if (lane == 0) bulk_wait_group_read<1>();
                __syncwarp();
              }
#pragma unroll 1
              for (int h = 0; h < Cfg::kCCols / 32; ++h) {
                const int cc = c0 + 32 * h;
                uint32_t r[32];
                __syncwarp();
                tmem_ld_x32(taddr + cc, r);
                tmem_ld_wait_x32(r);
                if (cc + 32 >= ncols) release_acc();
                const int n = n0 + cc;
                float f[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
                apply_epilogue_row<32>(f, p.tensor_scale, p.epilogue, p.bias, n);
                uint32_t wv[16];
                if (p.out_dtype == 0) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) {
                    const __nv_bfloat162 b2 = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
                    wv[j] = *reinterpret_cast<const uint32_t*>(&b2);
                  }
                } else {
#pragma unroll
                  for (int j = 0; j < 16; ++j) {
                    const __half2 h2 = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
                    wv[j] = *reinterpret_cast<const uint32_t*>(&h2);
                  }
                }
                // 16-byte piece q of this half: 128B swizzle (piece ^ row % 8) for 128-byte rows,
                // 64B swizzle (piece ^ (row / 2) % 4) for 64-byte rows
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const uint32_t off = Cfg::kCCols == 64
                                           ? lane * 128 + (((4 * h + q) ^ (lane & 7)) << 4)
                                           : lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4);
                  st_shared_v4(sb + off, wv[4 * q], wv[4 * q + 1], wv[4 * q + 2], wv[4 * q + 3]);
                }
              }
              fence_proxy_async_smem();  // the TMA store reads the staging through the async proxy
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tm_c, sb, n0 + c0, m0 + quarter * 32);
                bulk_commit_group();
              }
              ++c_stores;
            }
          } else {
            release_acc();
          }
          continue;
        }
      }
      if (warp_rows) {
        for (int c0 = 0; c0 < ncols; c0 += kEB) {
          uint32_t r[kEB];
          __syncwarp();
          tmem_ld_cols<kEB>(taddr + c0, r);
          tmem_ld_wait();
          if (!row_ok) continue;  // the warp meets again at the next __syncwarp
          float acc[kEB];
#pragma unroll
          for (int j = 0; j < kEB; ++j) acc[j] = __uint_as_float(r[j]);
          const int n = n0 + c0;
          const int64_t rowbase = static_cast<int64_t>(m) * p.N + n;
          if (p.split_k <= 1 && p.split_out == kOutAtomic) {
            float* o = reinterpret_cast<float*>(p.out) + rowbase;
#pragma unroll
            for (int j = 0; j < kEB; ++j) atomicAdd(o + j, acc[j] * p.tensor_scale);
          } else if (p.split_k <= 1) {
            apply_epilogue_row<kEB>(acc, p.tensor_scale, p.epilogue, p.bias, n);
            store_row<kEB>(p.out, rowbase, acc, p.out_dtype, p.vec_out);
          } else if (p.split_out == kOutPartial) {
            float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) +
                                                  static_cast<int64_t>(sg.z) * p.M * p.N + rowbase);
#pragma unroll
            for (int j = 0; j < kEB / 4; ++j)
              o[j] = make_float4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
          } else if (p.split_out == kOutPlane) {
#pragma unroll
            for (int j = 0; j < kEB; ++j) acc[j] *= p.tensor_scale;
            store_row<kEB>(p.out, static_cast<int64_t>(sg.z) * p.M * p.N + rowbase, acc,
                           p.out_dtype, p.vec_out);
          } else {
            float* o = reinterpret_cast<float*>(p.out) + rowbase;
#pragma unroll
            for (int j = 0; j < kEB; ++j) atomicAdd(o + j, acc[j] * p.tensor_scale);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (Cfg::kPair && rank != 0) mbar_arrive_remote(mapa_shared(smem_u32(&ctl.acc_empty), 0));
        else mbar_arrive(smem_u32(&ctl.acc_empty));
      }
    }
    // this warp's TMA stores of C complete before the grid does
    if (Cfg::kTmaStore && c_stores > 0 && lane == 0) bulk_wait_group_all();
  }

  // ------------------------------------------------------------------ teardown
  __syncwarp();  // lanes that skipped a role's single-thread loop meet their lane 0 here
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // tensor memory is freed only after every MMA the MMA thread issued is done (pairs: rank
    // 0's last commit arrives in both CTAs)
    if (lane == 0) mbar_wait(smem_u32(&ctl.drain), 0, p.err, kErrWaitMma, nullptr);
    __syncwarp();
    tc_fence_after();
    if constexpr (!Cfg::kPair) tmem_dealloc(tbase, Cfg::kTmemCols);
  }
  if constexpr (Cfg::kPair) {
    // neither CTA frees its tensor memory or exits while the peer may still arrive on its
    // barriers or store into its shared memory
    cluster_sync_all();
    if (warp == 1) tmem_dealloc_pair(tbase, Cfg::kTmemCols);
  }
}

// Stream-K fix-up as its own grid (tiles of 64 or 128 token rows): a split tile's partials
// are 32-128 KB per contributor and a tile can have ten contributors, more than one SM reads
// quickly from L2, so every split tile is summed by kFixupBlocks CTAs instead of by its last
// contributor. Same sums in the same (CTA) order as the in-kernel fix-up, so the same bits.
// Block b handles tile b / kFixupBlocks; tiles computed by one CTA were written by the GEMM.
constexpr int kFixupBlocks = 16;
constexpr int kFixupThreads = 256;

template <int BM>
__global__ void __launch_bounds__(kFixupThreads)
    streamk_fixup_kernel(const GemmParams p, int gemm_grid) {
  Schedule sch;
  sch.init(p, gemm_grid);
  Seg sg;
  sg.tile = blockIdx.x / kFixupBlocks;
  const int part = blockIdx.x % kFixupBlocks;
  const int first = sch.cta_of(sg.tile * p.nks);
  const int last = sch.cta_of((sg.tile + 1) * p.nks - 1);
  if (first == last) return;
  streamk_reduce<BM>(p, sch, sg, first, last, part * kFixupThreads + threadIdx.x,
                     kFixupBlocks * kFixupThreads);
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
      store_out(out, i * 4 + j, apply_epilogue(__fmul_rn(o[j], ts), epi, bias, n + j), dtype);
  }
}

}  // namespace bd
