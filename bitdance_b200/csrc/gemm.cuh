// gemm.cuh -- fused W4A6 GEMM for sm_100a: C = A_mxfp6 . transcode(B_nvfp4)^T.
//
// Tiles of C^T: 128 weight rows (N, the MMA's M operand) x BN tokens (M, the MMA's N
// operand), so a decode batch of a few tokens still fills 128-row MMAs.
//
// Persistent CTAs walk a schedule of "segments" (a tile and a range of 128-wide K chunks):
//   * stream-K (the default): the (tile, K chunk) units are cut into one contiguous range per
//     CTA; a tile split between CTAs is finished in-kernel -- every contributor stores its
//     fp32 partial in a per-CTA slot, the last one to arrive (atomic counter) sums the slots
//     in CTA order and writes C, so results do not depend on timing;
//   * explicit split-K (split_k >= 1): items (tile, split) dealt round-robin, written as
//     partial planes, fp32 workspace planes or fp32 atomics (the reference's split modes).
//
// Warp roles (704 threads):
//   warp 0      producer   TMA: packed NVFP4 codes (8 KB, 64B-swizzled), E4M3 scales (1 KB),
//                          token tile (128B-swizzled), token E8M0 scales; one mbarrier/stage.
//   warps 6..21 transcode  16 warps; warp (quarter q, K block j) turns rows 32q..32q+31 x
//                          32 K-elements into E4M3 bytes in tensor memory (tcgen05.st; the
//                          MMA reads its A operand from there) and their E8M0 scales.
//   warp 1      MMA        tcgen05.cp of both scale blocks, 4 block-scaled tcgen05.mma
//                          (kind::mxf8f6f4, A from TMEM, K = 32 each), commit frees the stage.
//   warps 2..5  epilogue   TMEM accumulator -> registers -> C / partials (double-buffered
//                          accumulators when tensor memory allows, so it overlaps the next
//                          segment's main loop).
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
constexpr int cpow2(int x) {
  int p = 32;
  while (p < x) p *= 2;
  return p;
}

template <int BN, int KS>
struct GemmCfg {
  // KS 128-wide K chunks per pipeline stage
  static constexpr int kStages = KS == 2 ? (BN >= 64 ? 3 : (BN >= 32 ? 4 : 5))
                                         : (BN >= 256 ? 4 : (BN >= 128 ? 5 : (BN >= 64 ? 6 : 8)));
  static constexpr int kTok = KS * BN * 128;     // token tiles (E2M3 operand image), SW128
  static constexpr int kWCode = KS * 128 * 64;   // packed NVFP4 codes, SW64
  static constexpr int kWScale = KS * 128 * 8;   // E4M3 per-16 scales
  static constexpr int kTokScale = cround(KS * BN * 4, 128);
  static constexpr int oTok = 0;
  static constexpr int oWCode = cround(oTok + kTok, 1024);
  static constexpr int oWScale = oWCode + kWCode;
  static constexpr int oTokScale = oWScale + kWScale;
  static constexpr int kStageBytes = cround(oTokScale + kTokScale, 1024);
  static constexpr int kTxBytes = kWCode + kWScale + kTok + KS * BN * 4;
  // tensor memory: accumulators | A operand (32 columns per chunk) | scale factors: per chunk
  // 4 columns of weight scales (quarter q uses column q) + BN/32 columns of token scales,
  // padded so every scale-factor address the MMA gets is a multiple of 4 columns
  static constexpr int kTokSfCols = BN >= 32 ? BN / 32 : 1;
  static constexpr int kSfColsPerChunk = 4 + cround(kTokSfCols, 4);
  // narrow tiles alternate two accumulators along K so consecutive MMAs do not wait on
  // each other's result; the epilogue adds them
  static constexpr int kChains = BN <= 64 ? 2 : 1;
  static constexpr int kAccCols = (kChains * BN) < 32 ? 32 : kChains * BN;
  static constexpr int kPerStageCols = KS * (32 + kSfColsPerChunk);
  static constexpr int kNumAcc = (2 * kAccCols + kStages * kPerStageCols <= 512) ? 2 : 1;
  static constexpr int kACol0 = kNumAcc * kAccCols;
  static constexpr int kSfCol0 = kACol0 + kStages * KS * 32;
  static constexpr int kTmemCols = cpow2(kSfCol0 + kStages * KS * kSfColsPerChunk);
  static constexpr int oCtl = kStages * kStageBytes;
  static constexpr int kCtlBytes = 2048;
  static constexpr int kSmemBytes = oCtl + kCtlBytes + 1024;  // + alignment slack
  static constexpr int kTranscodeWarps = 16;
  static constexpr int kEpiWarps = 4;
  static constexpr int kThreads = 32 * (2 + kEpiWarps + kTranscodeWarps);
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kTmemCols <= 512, "tensor memory budget");
  static_assert(kStages <= 8, "control block holds 8 stages");
  static_assert(kSfCol0 % 4 == 0 && kSfColsPerChunk % 4 == 0 && kACol0 % 8 == 0,
                "tensor-memory operand addresses stay 4-column aligned");
};

struct GemmCtl {
  uint64_t full[8], ready[8], empty[8], acc_full[2], acc_empty[2], drain;
  uint32_t tmem_base;
  uint32_t abort_flag;
  uint32_t bcast;
  TranscodeTables tab;
};

struct GemmParams {
  void* out;                    // C, or the fp32 workspace planes (kOutPartial)
  float* slots;                 // stream-K partial slots [grid][2][BN][128]
  uint32_t* counters;           // stream-K per-tile arrival counters (zero between calls)
  const __nv_bfloat16* bias;
  float tensor_scale;
  int M, N, K;
  int n_tiles, m_tiles, nks;    // nks: pipeline stages (KS chunks) per tile
  int split_k;                  // 0 = stream-K, else explicit split
  int split_out;                // output mode of explicit split segments
  int out_dtype, epilogue;
  uint32_t* err;
};

// One contiguous run of stages of one tile.
struct Seg {
  int tile, k0, k1, z, slot;  // slot: -1 full tile, 0/1 stream-K partial slot
};

// The work of CTA `c` of `G`: segment number `idx` (false when there is none). All indices
// fit 32 bits (the host rejects larger problems).
struct Schedule {
  int U;        // units (tile, stage)
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

__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Eight E2M1 nibbles (one word) -> eight E4M3 bytes (two words) with the magnitude table
// T of the 16-block's class. Signs: byte i of (w<<4) / w carries the sign of element 2i /
// 2i+1 in bit 7, so one prmt gathers four of them.
__device__ __forceinline__ void nib8_to_e4m3(uint32_t w, uint2 T, uint32_t& lo, uint32_t& hi) {
  const uint32_t m = w & 0x77777777u;
  const uint32_t t = w << 4;
  lo = (prmt(t, w, 0x5140u) & 0x80808080u) | prmt(T.x, T.y, m);
  hi = (prmt(t, w, 0x7362u) & 0x80808080u) | prmt(T.x, T.y, m >> 16);
}

// E8M0 byte of a 32-block from its two E4M3 scale bytes.
__device__ __forceinline__ uint32_t e8m0_of_pair(const TranscodeTables& t, uint32_t s0,
                                                 uint32_t s1) {
  const int e0 = t.info[s0 & 0x7Fu] >> 3, e1 = t.info[s1 & 0x7Fu] >> 3;
  return static_cast<uint32_t>(max(e0, e1) + 111);
}

template <int BN, int KS>
__global__ void __launch_bounds__(GemmCfg<BN, KS>::kThreads, 1)
    w4a6_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_as,
                     const __grid_constant__ CUtensorMap tm_w,
                     const __grid_constant__ CUtensorMap tm_ws, const GemmParams p) {
  using Cfg = GemmCfg<BN, KS>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  GemmCtl& ctl = *reinterpret_cast<GemmCtl*>(smem + Cfg::oCtl);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cta = blockIdx.x;
  volatile uint32_t* abort_flag = &ctl.abort_flag;
  Schedule sch;
  sch.init(p, gridDim.x);

  if (tid == 0) {
    ctl.abort_flag = 0;
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&ctl.full[s]), 1);
      mbar_init(smem_u32(&ctl.ready[s]), Cfg::kTranscodeWarps);
      mbar_init(smem_u32(&ctl.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&ctl.acc_full[b]), 1);
      mbar_init(smem_u32(&ctl.acc_empty[b]), Cfg::kEpiWarps);
    }
    mbar_init(smem_u32(&ctl.drain), 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_as);
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_ws);
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
      int i = 0;
      Seg sg;
      for (int idx = 0; sch.segment(cta, idx, sg) && !*abort_flag; ++idx) {
        const int mt = sg.tile / p.n_tiles, nt = sg.tile % p.n_tiles;
        for (int k = sg.k0; k < sg.k1; ++k, ++i) {
          const int s = i % S;
          const uint32_t ph = (i / S) & 1;
          if (!mbar_wait(smem_u32(&ctl.empty[s]), ph ^ 1u, p.err, kErrWaitEmpty, abort_flag)) break;
          uint8_t* st = smem + s * Cfg::kStageBytes;
          const uint32_t fb = smem_u32(&ctl.full[s]);
          const int kt = k * KS;
          const int32_t chunk = nt * (p.nks * KS) + kt;
          mbar_arrive_expect_tx(fb, Cfg::kTxBytes);
          tma_load_2d(smem_u32(st + Cfg::oWCode), &tm_w, 0, chunk * 128, fb);
          tma_load_2d(smem_u32(st + Cfg::oWScale), &tm_ws, 0, chunk, fb);
          tma_load_3d(smem_u32(st + Cfg::oTok), &tm_a, 0, mt * BN, kt, fb);
          tma_load_2d(smem_u32(st + Cfg::oTokScale), &tm_as, mt * BN, kt, fb);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int i = 0;
      Seg sg;
      for (int idx = 0; sch.segment(cta, idx, sg); ++idx) {
        const int buf = Cfg::kNumAcc == 2 ? (idx & 1) : 0;
        const uint32_t use = Cfg::kNumAcc == 2 ? (idx >> 1) : idx;
        if (!mbar_wait(smem_u32(&ctl.acc_empty[buf]), (use & 1) ^ 1u, p.err, kErrWaitAccum,
                       abort_flag))
          break;
        tc_fence_after();
        const uint32_t tD = tbase + buf * Cfg::kAccCols;
        bool ok = true;
        for (int k = sg.k0; k < sg.k1; ++k, ++i) {
          const int s = i % S;
          const uint32_t ph = (i / S) & 1;
          if (!mbar_wait(smem_u32(&ctl.ready[s]), ph, p.err, kErrWaitOperand, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t tok = smem_u32(smem + s * Cfg::kStageBytes + Cfg::oTok);
#pragma unroll
          for (int h = 0; h < KS; ++h) {
            const uint32_t tA = tbase + Cfg::kACol0 + (s * KS + h) * 32;
            const uint32_t tSfW = tbase + Cfg::kSfCol0 + (s * KS + h) * Cfg::kSfColsPerChunk;
            const uint32_t tSfA = tSfW + 4;
            const uint32_t ab = tok + h * BN * 128;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t idesc = idesc_mxf8f6f4(128, BN, kFmtE4M3, kFmtE2M3, kk, kk);
              const int chain = kk % Cfg::kChains;
              const bool first = (k == sg.k0 && h == 0 && kk < Cfg::kChains);
              mma_mxf8f6f4_ts(tD + chain * BN, tA + kk * 8, sdesc_sw128(ab + kk * 32), idesc,
                              tSfW, tSfA, first ? 0u : 1u);
            }
          }
          tc_commit(smem_u32(&ctl.empty[s]));
        }
        tc_commit(smem_u32(&ctl.acc_full[buf]));
        if (!ok) break;
      }
      // arrives once every tcgen05 operation this thread issued has completed
      tc_commit(smem_u32(&ctl.drain));
    }
  } else if (warp >= 2 + Cfg::kEpiWarps) {
    // ------------------------------------------------------------------ transcode
    // Software-pipelined by one stage: the tensor-memory stores of stage i drain while stage
    // i+1 is loaded and converted; only then does the warp wait for them and signal ready(i).
    // (Stage i+1's data never depends on ready(i): the producer is S >= 2 stages ahead.)
    const int tw = warp - 2 - Cfg::kEpiWarps;   // 0..15
    const int quarter = warp & 3;               // TMEM lane quarter this warp may access
    const int j = tw >> 2;                      // K block (32 elements) of each chunk
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = tbase + (static_cast<uint32_t>(quarter * 32) << 16);
    int i = 0, prev = -1;
    Seg sg;
    for (int idx = 0; sch.segment(cta, idx, sg) && !*abort_flag; ++idx) {
      for (int k = sg.k0; k < sg.k1; ++k, ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if (!mbar_wait(smem_u32(&ctl.full[s]), ph, p.err, kErrWaitTma, abort_flag)) break;
        const uint8_t* st = smem + s * Cfg::kStageBytes;
        uint32_t v[KS][8];
        uint32_t sfw_word[KS];
        uint32_t tok[KS][Cfg::kTokSfCols];
#pragma unroll
        for (int h = 0; h < KS; ++h) {
          // 64B-swizzled codes: 16-byte chunk c of row r at r*64 + (c ^ ((r >> 1) & 3)) * 16
          const uint4 q = *reinterpret_cast<const uint4*>(
              st + Cfg::oWCode + h * 8192 + row * 64 + ((j ^ ((row >> 1) & 3)) << 4));
          const uint8_t* srow = st + Cfg::oWScale + h * 1024 + row * 8;
          const uint32_t sc = *reinterpret_cast<const uint16_t*>(srow + j * 2);
          uint2 T0, T1;
          uint32_t e8;
          scale_pair(ctl.tab, sc & 0xFFu, sc >> 8, T0, T1, e8);
          nib8_to_e4m3(q.x, T0, v[h][0], v[h][1]);
          nib8_to_e4m3(q.y, T0, v[h][2], v[h][3]);
          nib8_to_e4m3(q.z, T1, v[h][4], v[h][5]);
          nib8_to_e4m3(q.w, T1, v[h][6], v[h][7]);
          if (j == 0) {
            // weight scales of this row's four K blocks, one word for column sfw + quarter
            const uint2 all = *reinterpret_cast<const uint2*>(srow);
            sfw_word[h] = e8m0_of_pair(ctl.tab, all.x & 0xFFu, (all.x >> 8) & 0xFFu) |
                          (e8m0_of_pair(ctl.tab, (all.x >> 16) & 0xFFu, all.x >> 24) << 8) |
                          (e8m0_of_pair(ctl.tab, all.y & 0xFFu, (all.y >> 8) & 0xFFu) << 16) |
                          (e8m0_of_pair(ctl.tab, (all.y >> 16) & 0xFFu, all.y >> 24) << 24);
          } else if (j == 1) {
            // token scales: token n = lane + 32c at column c, in every lane quarter
            const uint32_t* raw = reinterpret_cast<const uint32_t*>(st + Cfg::oTokScale) + h * BN;
#pragma unroll
            for (int c = 0; c < Cfg::kTokSfCols; ++c)
              tok[h][c] = (lane + 32 * c < BN) ? raw[lane + 32 * c] : 0u;
          }
        }
        if (prev >= 0) {
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&ctl.ready[prev]));
        }
#pragma unroll
        for (int h = 0; h < KS; ++h) {
          tmem_st_x8(lane_base + Cfg::kACol0 + (s * KS + h) * 32 + j * 8, v[h]);
          const uint32_t sfw = Cfg::kSfCol0 + (s * KS + h) * Cfg::kSfColsPerChunk;
          if (j == 0) {
            tmem_st_x1(lane_base + sfw + quarter, sfw_word[h]);
          } else if (j == 1) {
            if constexpr (Cfg::kTokSfCols == 1) {
              tmem_st_x1(lane_base + sfw + 4, tok[h][0]);
            } else if constexpr (Cfg::kTokSfCols == 2) {
              tmem_st_x2(lane_base + sfw + 4, tok[h][0], tok[h][1]);
            } else if constexpr (Cfg::kTokSfCols == 4) {
              tmem_st_x4(lane_base + sfw + 4, tok[h][0], tok[h][1], tok[h][2], tok[h][3]);
            } else {
              uint32_t t8[8];
#pragma unroll
              for (int c = 0; c < 8; ++c) t8[c] = tok[h][c % Cfg::kTokSfCols];
              tmem_st_x8(lane_base + sfw + 4, t8);
            }
          }
        }
        prev = s;
      }
    }
    if (prev >= 0) {
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.ready[prev]));
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    // accumulator columns per tensor-memory load
    constexpr int kB = (BN < 32 || Cfg::kChains == 2) ? 16 : 32;
    const int quarter = warp & 3;
    const int ep_tid = tid - 64;  // 0..127
    Seg sg;
    for (int idx = 0; sch.segment(cta, idx, sg); ++idx) {
      const int buf = Cfg::kNumAcc == 2 ? (idx & 1) : 0;
      const uint32_t use = Cfg::kNumAcc == 2 ? (idx >> 1) : idx;
      if (!mbar_wait(smem_u32(&ctl.acc_full[buf]), use & 1, p.err, kErrWaitAccum, abort_flag))
        break;
      tc_fence_after();
      const int mt = sg.tile / p.n_tiles, nt = sg.tile % p.n_tiles;
      const int n = nt * 128 + quarter * 32 + lane;
      const int m0 = mt * BN;
      const int mcols = min(BN, p.M - m0);  // valid token columns of this tile
      const uint32_t taddr =
          tbase + buf * Cfg::kAccCols + (static_cast<uint32_t>(quarter * 32) << 16);
      const int row = quarter * 32 + lane;
      // accumulator columns [c0, c0 + kB) of this thread's row, chains added
      auto load_acc = [&](int c0, float (&acc)[kB]) {
        uint32_t r[kB];
        if constexpr (kB == 16) tmem_ld_x16(taddr + c0, r); else tmem_ld_x32(taddr + c0, r);
        if constexpr (Cfg::kChains == 2) {
          uint32_t r2[kB];
          if constexpr (kB == 16) tmem_ld_x16(taddr + BN + c0, r2);
          else tmem_ld_x32(taddr + BN + c0, r2);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < kB; ++jj) acc[jj] = __uint_as_float(r[jj]) + __uint_as_float(r2[jj]);
        } else {
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < kB; ++jj) acc[jj] = __uint_as_float(r[jj]);
        }
      };
      bool finish = false;
      int first = 0, last = -1;
      if (sg.slot >= 0) {
        // stream-K partial: store the slot, then count arrivals for this tile
        float* slot = p.slots + (static_cast<int64_t>(cta) * 2 + sg.slot) * (BN * 128);
        for (int c0 = 0; c0 < mcols; c0 += kB) {
          float acc[kB];
          load_acc(c0, acc);
#pragma unroll
          for (int jj = 0; jj < kB; ++jj) __stcg(slot + (c0 + jj) * 128 + row, acc[jj]);
        }
        __threadfence();
        first = sch.cta_of(sg.tile * p.nks);
        last = sch.cta_of((sg.tile + 1) * p.nks - 1);
        named_barrier(1, 32 * Cfg::kEpiWarps);
        if (ep_tid == 0) {
          const uint32_t old = atomicAdd(p.counters + sg.tile, 1u);
          const bool fin = old == static_cast<uint32_t>(last - first);
          if (fin) p.counters[sg.tile] = 0;  // every contributor has arrived: rearm
          ctl.bcast = fin ? 1u : 0u;
        }
        named_barrier(1, 32 * Cfg::kEpiWarps);
        finish = ctl.bcast != 0;
        named_barrier(1, 32 * Cfg::kEpiWarps);
        if (finish) __threadfence();
      }
      if (sg.slot < 0 || finish) {
        for (int c0 = 0; c0 < mcols; c0 += kB) {
          float acc[kB];
          load_acc(c0, acc);   // this CTA's own part straight from tensor memory
          if (finish) {
            // add the contributors in CTA order (own part in its place): the result does not
            // depend on which CTA happened to arrive last
            float own[kB];
#pragma unroll
            for (int jj = 0; jj < kB; ++jj) {
              own[jj] = acc[jj];
              acc[jj] = 0.0f;
            }
            for (int c = first; c <= last; ++c) {
              if (c == cta) {
#pragma unroll
                for (int jj = 0; jj < kB; ++jj) acc[jj] += own[jj];
                continue;
              }
              const int sl = (sch.u0(c) / p.nks == sg.tile) ? 0 : 1;
              const float* slot = p.slots + (static_cast<int64_t>(c) * 2 + sl) * (BN * 128);
#pragma unroll
              for (int jj = 0; jj < kB; ++jj) acc[jj] += __ldcg(slot + (c0 + jj) * 128 + row);
            }
          }
#pragma unroll
          for (int jj = 0; jj < kB; ++jj) {
            const int m = m0 + c0 + jj;
            if (c0 + jj < mcols) {
              const float a = acc[jj];
              if (p.split_k == 0 || p.split_k == 1) {
                if (p.split_out == kOutAtomic) {
                  atomicAdd(reinterpret_cast<float*>(p.out) + static_cast<int64_t>(m) * p.N + n,
                            a * p.tensor_scale);
                } else {
                  store_out(p.out, static_cast<int64_t>(m) * p.N + n,
                            apply_epilogue(a * p.tensor_scale, p.epilogue, p.bias, n),
                            p.out_dtype);
                }
              } else if (p.split_out == kOutPartial) {
                reinterpret_cast<float*>(p.out)[(static_cast<int64_t>(sg.z) * p.M + m) * p.N + n] = a;
              } else if (p.split_out == kOutPlane) {
                store_out(p.out, (static_cast<int64_t>(sg.z) * p.M + m) * p.N + n,
                          a * p.tensor_scale, p.out_dtype);
              } else {
                atomicAdd(reinterpret_cast<float*>(p.out) + static_cast<int64_t>(m) * p.N + n,
                          a * p.tensor_scale);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.acc_empty[buf]));
    }
  }

  // ------------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    // tensor memory is freed only after every MMA the MMA thread issued is done
    if (lane == 0) mbar_wait(smem_u32(&ctl.drain), 0, p.err, kErrWaitMma, nullptr);
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
