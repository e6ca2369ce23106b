// bitdance.cu -- the C ABI of the library (include/bitdance_b200.h): argument checks,
// tensor-map set-up and launches of the kernels in transcode.cuh and gemm.cuh.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/bitdance_b200.h"
#include "gemm.cuh"
#include "probe.cuh"
#include "quantize_b.cuh"
#include "sm100.cuh"
#include "transcode.cuh"

namespace bd {

// Error word that kernels OR their error bits into (one per device that loads the library).
__device__ uint32_t g_err_word;

namespace {

constexpr int kMaxDevices = 64;

inline cudaStream_t as_stream(bd_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// Per-device facts, computed once.
struct DeviceInfo {
  int sm_count = 0;
  bool is_sm100 = false;
  uint32_t* err = nullptr;
  bool ready = false;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(DeviceInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BD_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return BD_ERR_CUDA;
    d.is_sm100 = (major == 10 && minor == 0);
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_err_word) != cudaSuccess) return BD_ERR_CUDA;
    d.err = static_cast<uint32_t*>(p);
    d.ready = true;
  }
  *out = &d;
  return d.is_sm100 ? BD_OK : BD_ERR_ARCH;
}

// Diagnostic of the bounded waits: warp 0 waits on an mbarrier that nothing arrives at, with
// a limit of `limit` cycles, and so records kErrWaitTma and raises the abort flag; warp 1 waits
// on another such barrier with the GEMM's default limit and must leave through that flag.
// The same mbar_wait as the GEMM's roles; it ends with a status, not a hung context.
__global__ void wait_selftest_kernel(uint32_t* err, unsigned long long limit) {
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bars[0]), 1);
    mbar_init(smem_u32(&bars[1]), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    if (warp == 0)
      mbar_wait(smem_u32(&bars[0]), 0, err, kErrWaitTma, &abort_flag, limit);
    else
      mbar_wait(smem_u32(&bars[1]), 0, err, kErrWaitOperand, &abort_flag);
  }
  __syncwarp();
}

// Scratch of bd_w4a6_gemm_noalloc: the stream-K partial slots and per-tile counters of one
// call live in this file-scope array instead of a caller-provided workspace, so that entry
// point performs no device allocation. 16 MiB holds the stream-K scratch of every problem
// with at most 32 token rows per tile on a 148-SM B200 (148 x 2 x 32 x 256 fp32 slots plus
// counters); larger problems that need stream-K scratch are rejected.
constexpr size_t kNoAllocScratchBytes = size_t{16} << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device, with
// that device current).
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BD_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_dev_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return BD_ERR_CUDA;
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return BD_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda needed).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

bool make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, void* base, uint64_t d0, uint64_t d1,
                 uint64_t stride1_bytes, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[2] = {d0, d1};
  const cuuint64_t strides[1] = {stride1_bytes};
  const cuuint32_t box[2] = {b0, b1};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_3d(CUtensorMap* m, CUtensorMapDataType dt, void* base, uint64_t d0, uint64_t d1,
                 uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0,
                 uint32_t b1, uint32_t b2, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, dt, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int grid_for(int64_t work, int per_block, const DeviceInfo* d) {
  int64_t blocks = (work + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(d->sm_count) * 8;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

// Token rows loaded per tile (the MMA's M operand is 128 rows; a decode batch loads fewer).
int token_tile(int M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  return 128;
}

// Stream-K scratch of one call: per-CTA partial slots [grid][2][BM][256] fp32, then one
// arrival counter per tile. Counters must be zero before the first call; every call leaves
// them zero again.
struct StreamKSizes {
  size_t slots_bytes, counter_bytes, total;
};
StreamKSizes streamk_sizes(int M, int N, int K, int sm_count) {
  const int bm = token_tile(M);
  const int64_t tiles = static_cast<int64_t>((N + kTileN - 1) / kTileN) * ((M + bm - 1) / bm);
  const int64_t units = tiles * (K / 128);
  const int64_t grid = units < sm_count ? units : sm_count;
  StreamKSizes z;
  z.slots_bytes =
      (static_cast<size_t>(grid) * 2 * bm * kTileN * sizeof(float) + 255) / 256 * 256;
  z.counter_bytes = (static_cast<size_t>(tiles) * sizeof(uint32_t) + 255) / 256 * 256;
  z.total = z.slots_bytes + z.counter_bytes;
  return z;
}

struct GemmMaps {
  CUtensorMap a, as, w, ws, c;  // c: 16-bit C for TMA stores (GemmParams::tma_c), else zeros
};

template <int BM, bool kClassWords>
int launch_gemm(const GemmMaps& m, const GemmParams& p, int grid, bool overlap,
                cudaStream_t stream) {
  using Cfg = GemmCfg<BM>;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    if (cudaFuncSetAttribute(w4a6_gemm_kernel<BM, kClassWords>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Cfg::kSmemBytes) != cudaSuccess)
      return BD_ERR_CUDA;
    configured.fetch_or(bit);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (overlap) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (Cfg::kPair) {  // clusters of two CTAs (grid is even)
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 2;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  if (cudaLaunchKernelEx(&cfg, w4a6_gemm_kernel<BM, kClassWords>, m.a, m.as, m.w, m.ws, m.c, p) !=
      cudaSuccess)
    return BD_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

template <bool kClassWords>
int launch_gemm_bm(int bm, const GemmMaps& m, const GemmParams& p, int grid, bool overlap,
                   cudaStream_t s) {
  switch (bm) {
    case 16: return launch_gemm<16, kClassWords>(m, p, grid, overlap, s);
    case 32: return launch_gemm<32, kClassWords>(m, p, grid, overlap, s);
    case 64: return launch_gemm<64, kClassWords>(m, p, grid, overlap, s);
    case 256: return launch_gemm<256, kClassWords>(m, p, grid, overlap, s);
    default: return launch_gemm<128, kClassWords>(m, p, grid, overlap, s);
  }
}

int launch_gemm_any(int bm, bool class_words, const GemmMaps& m, const GemmParams& p, int grid,
                    bool overlap, cudaStream_t s) {
  return class_words ? launch_gemm_bm<true>(bm, m, p, grid, overlap, s)
                     : launch_gemm_bm<false>(bm, m, p, grid, overlap, s);
}

// The stream-K fix-up grid of 64- and 128-row token tiles (GemmParams::fixup_kernel), after the
// GEMM on the same stream.
int launch_fixup(int bm, const GemmParams& p, int64_t tiles, int gemm_grid, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(tiles * kFixupBlocks));
  if (bm == 64)
    streamk_fixup_kernel<64><<<grid, kFixupThreads, 0, s>>>(p, gemm_grid);
  else
    streamk_fixup_kernel<128><<<grid, kFixupThreads, 0, s>>>(p, gemm_grid);
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

}  // namespace
}  // namespace bd

using namespace bd;

extern "C" {

int bd_version(void) { return 100; }

const char* bd_status_string(int status) {
  switch (status) {
    case BD_OK: return "ok";
    case BD_ERR_INVALID_ARG: return "invalid argument";
    case BD_ERR_SHAPE: return "unsupported shape";
    case BD_ERR_ALIGNMENT: return "misaligned pointer";
    case BD_ERR_ARCH: return "device is not sm_100 (B200)";
    case BD_ERR_CUDA: return "CUDA runtime error";
    case BD_ERR_WORKSPACE: return "workspace missing or too small";
    case BD_ERR_DEVICE: return "a kernel reported an error";
    default: return "unknown status";
  }
}

int bd_device_error(uint32_t* word, int clear) {
  if (word == nullptr) return BD_ERR_INVALID_ARG;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  if (cudaDeviceSynchronize() != cudaSuccess) return BD_ERR_CUDA;
  if (cudaMemcpy(word, d->err, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess)
    return BD_ERR_CUDA;
  if (clear && cudaMemset(d->err, 0, sizeof(uint32_t)) != cudaSuccess) return BD_ERR_CUDA;
  return BD_OK;
}

int bd_selftest_bounded_wait(int64_t limit_cycles, bd_stream_t stream) {
  if (limit_cycles < 1000 || static_cast<unsigned long long>(limit_cycles) > kWaitLimitCycles)
    return BD_ERR_INVALID_ARG;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  wait_selftest_kernel<<<1, 64, 0, as_stream(stream)>>>(
      d->err, static_cast<unsigned long long>(limit_cycles));
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

int bd_probe_mma_peak(int64_t mmas_per_cta, int n_cols, int a_from_tmem, bd_stream_t stream) {
  if (mmas_per_cta < 1 || mmas_per_cta > (int64_t{1} << 21)) return BD_ERR_INVALID_ARG;
  if (n_cols < 16 || n_cols > 256 || n_cols % 16) return BD_ERR_INVALID_ARG;
  if (a_from_tmem < 0 || a_from_tmem > 2 || (a_from_tmem == 2 && n_cols != 256))
    return BD_ERR_INVALID_ARG;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    if (cudaFuncSetAttribute(mma_peak_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kProbeSmem) != cudaSuccess ||
        cudaFuncSetAttribute(mma_peak_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kProbeSmem) != cudaSuccess)
      return BD_ERR_CUDA;
    configured.fetch_or(bit);
  }
  if (a_from_tmem == 2) {  // CTA pairs: one cluster of two CTAs per pair of SMs
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(d->sm_count / 2 * 2));
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = kProbeSmem;
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, mma_peak_pair_kernel, static_cast<long long>(mmas_per_cta),
                           d->err) != cudaSuccess)
      return BD_ERR_CUDA;
    return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
  }
  mma_peak_kernel<<<d->sm_count, 128, kProbeSmem, as_stream(stream)>>>(
      static_cast<long long>(mmas_per_cta), n_cols, a_from_tmem ? 1 : 0, d->err);
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

int bd_transcode_nvfp4_to_mxfp6(const uint8_t* codes, const uint8_t* scales, uint8_t* e2m3_out,
                                uint8_t* e8m0_out, int64_t nblk32, int scale_block,
                                bd_stream_t stream) {
  if (scale_block != 16 && scale_block != 32) return BD_ERR_INVALID_ARG;
  if (nblk32 < 0) return BD_ERR_SHAPE;
  if (nblk32 == 0) return BD_OK;
  if (!codes || !scales || !e2m3_out || !e8m0_out) return BD_ERR_INVALID_ARG;
  if (!aligned(codes, 16) || !aligned(e2m3_out, 16) || (scale_block == 16 && !aligned(scales, 2)))
    return BD_ERR_ALIGNMENT;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  const int64_t stages = (nblk32 + kTxBlocks - 1) / kTxBlocks;
  const int grid = static_cast<int>(std::min<int64_t>(stages, static_cast<int64_t>(d->sm_count) * 4));
  const uint8_t* cb = reinterpret_cast<const uint8_t*>(codes);
  if (scale_block == 16)
    transcode_kernel<16><<<grid, kTxThreads, 0, as_stream(stream)>>>(
        cb, scales, reinterpret_cast<uint4*>(e2m3_out), e8m0_out, nblk32, d->err);
  else
    transcode_kernel<32><<<grid, kTxThreads, 0, as_stream(stream)>>>(
        cb, scales, reinterpret_cast<uint4*>(e2m3_out), e8m0_out, nblk32, d->err);
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

static int pack_b(const uint8_t* codes, const uint8_t* scales16, uint8_t* codes_tiled,
                  uint8_t* scales_tiled, int N, int K, bool class_words, bd_stream_t stream) {
  if (!codes || !scales16 || !codes_tiled || !scales_tiled) return BD_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0 || N % 128 || K % 128) return BD_ERR_SHAPE;
  if (!aligned(codes, 16) || !aligned(codes_tiled, 16) || !aligned(scales16, 8) ||
      !aligned(scales_tiled, 8))
    return BD_ERR_ALIGNMENT;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  const int64_t work = static_cast<int64_t>(N) * (K / 128);
  if (class_words)
    pack_b_kernel<true><<<grid_for(work, 256, d), 256, 0, as_stream(stream)>>>(
        codes, scales16, codes_tiled, scales_tiled, N, K);
  else
    pack_b_kernel<false><<<grid_for(work, 256, d), 256, 0, as_stream(stream)>>>(
        codes, scales16, codes_tiled, scales_tiled, N, K);
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

int bd_pack_b(const uint8_t* codes, const uint8_t* scales16, uint8_t* codes_tiled,
              uint8_t* scales_tiled, int N, int K, bd_stream_t stream) {
  return pack_b(codes, scales16, codes_tiled, scales_tiled, N, K, true, stream);
}

int bd_pack_b_e4m3(const uint8_t* codes, const uint8_t* scales16, uint8_t* codes_tiled,
                   uint8_t* scales_tiled, int N, int K, bd_stream_t stream) {
  return pack_b(codes, scales16, codes_tiled, scales_tiled, N, K, false, stream);
}

int bd_scales_e8m0_to_e4m3_pairs(const uint8_t* e8m0, uint8_t* e4m3_pairs, int64_t nblk32,
                                  bd_stream_t stream) {
  if (nblk32 < 0) return BD_ERR_SHAPE;
  if (nblk32 == 0) return BD_OK;
  if (!e8m0 || !e4m3_pairs) return BD_ERR_INVALID_ARG;
  if (!aligned(e4m3_pairs, 2)) return BD_ERR_ALIGNMENT;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  e8m0_to_e4m3_pairs_kernel<<<grid_for(nblk32, 256, d), 256, 0, as_stream(stream)>>>(
      e8m0, reinterpret_cast<uint16_t*>(e4m3_pairs), nblk32, d->err);
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

int bd_pack_a(const uint8_t* codes, const uint8_t* e8m0, uint8_t* a_packed, uint8_t* scales_tiled,
              int M, int K, bd_stream_t stream) {
  if (!codes || !e8m0 || !a_packed || !scales_tiled) return BD_ERR_INVALID_ARG;
  if (M <= 0 || K <= 0 || K % 128) return BD_ERR_SHAPE;
  if (!aligned(codes, 16) || !aligned(a_packed, 16) || !aligned(scales_tiled, 4))
    return BD_ERR_ALIGNMENT;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  // the natural codes are already the operand layout (the GEMM ignores bits 6..7): with
  // a_packed == codes only the scales are re-laid out
  const int64_t nchunks = static_cast<int64_t>(M) * K / 16;
  if (a_packed != codes)
    pack_a_codes_kernel<<<grid_for(nchunks, 256, d), 256, 0, as_stream(stream)>>>(codes, a_packed,
                                                                                   nchunks);
  const int Mp4 = (M + 3) / 4 * 4;
  const int64_t words = static_cast<int64_t>(K / 128) * Mp4;
  pack_a_scales_kernel<<<grid_for(words, 256, d), 256, 0, as_stream(stream)>>>(e8m0, scales_tiled,
                                                                                M, Mp4, K);
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

int bd_quantize_a_mxfp6(const void* x, int x_dtype, uint8_t* codes, uint8_t* e8m0,
                        uint8_t* scales_tiled, int M, int K, bd_stream_t stream) {
  return bd_quantize_a_mxfp6_ex(x, x_dtype, codes, e8m0, scales_tiled, M, K, 0u, stream);
}

int bd_quantize_a_mxfp6_ex(const void* x, int x_dtype, uint8_t* codes, uint8_t* e8m0,
                           uint8_t* scales_tiled, int M, int K, unsigned flags,
                           bd_stream_t stream) {
  if (flags & ~static_cast<unsigned>(BD_GEMM_OVERLAP_PREV)) return BD_ERR_INVALID_ARG;
  if (x_dtype != BD_IN_F32 && x_dtype != BD_IN_BF16) return BD_ERR_INVALID_ARG;
  if (!x || !codes || (!e8m0 && !scales_tiled)) return BD_ERR_INVALID_ARG;
  if (M <= 0 || K <= 0 || K % 32 || (scales_tiled && K % 128)) return BD_ERR_SHAPE;
  if (M > (1 << 30) / 4 || K > (1 << 24)) return BD_ERR_SHAPE;
  if (static_cast<int64_t>(M) * K >= (int64_t{1} << 36)) return BD_ERR_SHAPE;  // block ids in 31 bits
  if (!aligned(x, 16) || !aligned(codes, 16) || (scales_tiled && !aligned(scales_tiled, 4)))
    return BD_ERR_ALIGNMENT;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  const bool bf16 = x_dtype == BD_IN_BF16;
  const uint64_t nblk = static_cast<uint64_t>(M) * static_cast<uint64_t>(K / 32);
  const uint32_t row_bytes = bf16 ? QuantCfg<true>::kRowBytes : QuantCfg<false>::kRowBytes;
  // one 32-element block per row; the kernel's stages are boxes of kQRows rows
  CUtensorMap map;
  if (!make_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, const_cast<void*>(x), row_bytes, nblk,
                   row_bytes, row_bytes, kQRows,
                   bf16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B))
    return BD_ERR_CUDA;
  const int smem = bf16 ? QuantCfg<true>::kSmemBytes : QuantCfg<false>::kSmemBytes;
  const int per_sm = bf16 ? QuantCfg<true>::kCtasPerSm : QuantCfg<false>::kCtasPerSm;
  {
    static std::atomic<uint64_t> configured{0};
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = (1ull << (dev & 31)) << (bf16 ? 32 : 0);
    if (!(configured.load() & bit)) {
      const cudaError_t e =
          bf16 ? cudaFuncSetAttribute(quantize_a_kernel<true>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem)
               : cudaFuncSetAttribute(quantize_a_kernel<false>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return BD_ERR_CUDA;
      configured.fetch_or(bit);
    }
  }
  const int64_t stages = static_cast<int64_t>((nblk + kQRows - 1) / kQRows);
  const int grid = static_cast<int>(
      std::min<int64_t>(stages, static_cast<int64_t>(d->sm_count) * per_sm));
  const int Mp4 = (M + 3) / 4 * 4;
  // floor(2^64 / (K / 128)) + 1: chunk -> row by a multiply-high in the kernel
  const uint64_t nkt = static_cast<uint64_t>(K / 128 > 0 ? K / 128 : 1);
  const uint64_t nkt_magic = nkt > 1 ? ~0ull / nkt + 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kQThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (flags & BD_GEMM_OVERLAP_PREV) ? 1 : 0;
  const cudaError_t e =
      bf16 ? cudaLaunchKernelEx(&cfg, quantize_a_kernel<true>, map, codes, e8m0, scales_tiled, M,
                                K, Mp4, nkt_magic, d->err)
           : cudaLaunchKernelEx(&cfg, quantize_a_kernel<false>, map, codes, e8m0, scales_tiled, M,
                                K, Mp4, nkt_magic, d->err);
  if (e != cudaSuccess) return BD_ERR_CUDA;
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

int bd_quantize_b_nvfp4(const void* w, int w_dtype, uint8_t* codes, uint8_t* scales16,
                        uint32_t* tstat, int N, int K, bd_stream_t stream) {
  if (w_dtype != BD_IN_F32 && w_dtype != BD_IN_BF16) return BD_ERR_INVALID_ARG;
  if (!w || !codes || !scales16 || !tstat) return BD_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0 || K % 16) return BD_ERR_SHAPE;
  if (static_cast<int64_t>(N) * K >= (int64_t{1} << 38)) return BD_ERR_SHAPE;
  if (!aligned(w, 16) || !aligned(codes, 8) || !aligned(tstat, 4)) return BD_ERR_ALIGNMENT;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  const bool bf16 = w_dtype == BD_IN_BF16;
  const int64_t nblk = static_cast<int64_t>(N) * (K / 16);
  const int64_t nvec = nblk * (bf16 ? 2 : 4);
  cudaStream_t s = as_stream(stream);
  if (cudaMemsetAsync(tstat, 0, 2 * sizeof(uint32_t), s) != cudaSuccess) return BD_ERR_CUDA;
  const uint4* wv = static_cast<const uint4*>(w);
  const uint8_t* wb = static_cast<const uint8_t*>(w);
  if (bf16) {
    weight_amax_kernel<true><<<grid_for(nvec, 256, d), 256, 0, s>>>(wv, nvec, tstat, d->err);
    quantize_b_kernel<true><<<grid_for(nblk, 256, d), 256, 0, s>>>(wb, codes, scales16, nblk,
                                                                    tstat);
  } else {
    weight_amax_kernel<false><<<grid_for(nvec, 256, d), 256, 0, s>>>(wv, nvec, tstat, d->err);
    quantize_b_kernel<false><<<grid_for(nblk, 256, d), 256, 0, s>>>(wb, codes, scales16, nblk,
                                                                     tstat);
  }
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

size_t bd_query_workspace(int M, int N, int K, int split_k, int split_mode) {
  if (M <= 0 || N <= 0 || K <= 0 || N % 128 || K % 128 || split_k < 0) return 0;
  if (split_k == 0) {
    DeviceInfo* d = nullptr;
    const int st = device_info(&d);
    const int sms = (st == BD_OK || st == BD_ERR_ARCH) && d ? d->sm_count : 148;
    return streamk_sizes(M, N, K, sms > 0 ? sms : 148).total;
  }
  if (split_k <= 1 || split_mode != BD_SPLIT_REDUCE) return 0;
  return static_cast<size_t>(split_k) * static_cast<size_t>(M) * static_cast<size_t>(N) *
         sizeof(float);
}

int bd_splitk_reduce(const float* partials, void* c, const void* bias, float b_tensor_scale,
                     int M, int N, int split_k, int out_dtype, int epilogue, bd_stream_t stream) {
  if (!partials || !c) return BD_ERR_INVALID_ARG;
  if (out_dtype < BD_OUT_BF16 || out_dtype > BD_OUT_F32) return BD_ERR_INVALID_ARG;
  if (epilogue < BD_EPI_NONE || epilogue > BD_EPI_BIAS_GELU) return BD_ERR_INVALID_ARG;
  if (epilogue != BD_EPI_NONE && !bias) return BD_ERR_INVALID_ARG;
  if (M <= 0 || N <= 0 || N % 4 || split_k < 1) return BD_ERR_SHAPE;
  if (!aligned(partials, 16)) return BD_ERR_ALIGNMENT;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  const int64_t work = static_cast<int64_t>(M) * N / 4;
  splitk_reduce_kernel<<<grid_for(work, 256, d), 256, 0, as_stream(stream)>>>(
      partials, c, static_cast<const __nv_bfloat16*>(bias), b_tensor_scale, M, N, split_k,
      out_dtype, epilogue);
  return cudaPeekAtLastError() == cudaSuccess ? BD_OK : BD_ERR_CUDA;
}

int bd_w4a6_gemm(void* c, const uint8_t* a, const uint8_t* a_scales, const uint8_t* b,
                 const uint8_t* b_scales, float b_tensor_scale, const void* bias, int M, int N,
                 int K, int split_k, int split_mode, int out_dtype, int epilogue, void* workspace,
                 size_t workspace_bytes, bd_stream_t stream) {
  return bd_w4a6_gemm_ex(c, a, a_scales, b, b_scales, b_tensor_scale, bias, M, N, K, split_k,
                         split_mode, out_dtype, epilogue, workspace, workspace_bytes, 0u, stream);
}

int bd_w4a6_gemm_ex(void* c, const uint8_t* a, const uint8_t* a_scales, const uint8_t* b,
                    const uint8_t* b_scales, float b_tensor_scale, const void* bias, int M, int N,
                    int K, int split_k, int split_mode, int out_dtype, int epilogue,
                    void* workspace, size_t workspace_bytes, unsigned flags, bd_stream_t stream) {
  if (flags & ~static_cast<unsigned>(BD_GEMM_OVERLAP_PREV | BD_GEMM_WEIGHTS_STATIC |
                                     BD_GEMM_B_E4M3 | BD_GEMM_SINGLE_CTA))
    return BD_ERR_INVALID_ARG;
  if (!c || !a || !a_scales || !b || !b_scales) return BD_ERR_INVALID_ARG;
  if (out_dtype < BD_OUT_BF16 || out_dtype > BD_OUT_F32) return BD_ERR_INVALID_ARG;
  if (epilogue < BD_EPI_NONE || epilogue > BD_EPI_BIAS_GELU) return BD_ERR_INVALID_ARG;
  if (epilogue != BD_EPI_NONE && !bias) return BD_ERR_INVALID_ARG;
  if (split_mode < BD_SPLIT_REDUCE || split_mode > BD_SPLIT_ATOMIC) return BD_ERR_INVALID_ARG;
  if (M <= 0 || N <= 0 || K <= 0 || N % 128 || K % 128) return BD_ERR_SHAPE;
  if (M > (1 << 30) / 4 || K > (1 << 24) || N > (1 << 24)) return BD_ERR_SHAPE;
  if (!aligned(a, 16) || !aligned(a_scales, 16) || !aligned(b, 16) || !aligned(b_scales, 16) ||
      (bias && !aligned(bias, 2)))
    return BD_ERR_ALIGNMENT;
  const int nkt = K / 128;
  if (split_k < 0 || (split_k > 0 && nkt % split_k)) return BD_ERR_SHAPE;
  if (split_mode == BD_SPLIT_ATOMIC && (out_dtype != BD_OUT_F32 || epilogue != BD_EPI_NONE))
    return BD_ERR_INVALID_ARG;
  if (split_k > 1 && split_mode == BD_SPLIT_PLANES && epilogue != BD_EPI_NONE)
    return BD_ERR_INVALID_ARG;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;

  int bm = token_tile(M);
  int m_tiles = (M + bm - 1) / bm;
  int n_tiles = (N + kTileN - 1) / kTileN;
  int64_t tiles = static_cast<int64_t>(m_tiles) * n_tiles;
  // split_k == 0: stream-K when the tiles do not fill the machine twice over, whole tiles
  // dealt round-robin otherwise (no fix-up needed); atomics never need the fix-up either
  const bool streamk = split_k == 0 && split_mode != BD_SPLIT_ATOMIC && tiles < 2 * d->sm_count;
  if (split_k == 0 && !streamk) split_k = 1;
  // whole 128-token tiles, N % 256 == 0: tiles of 256 tokens computed by CTA pairs
  const bool pair = bm == 128 && !streamk && split_k == 1 && split_mode != BD_SPLIT_ATOMIC &&
                    N % 256 == 0 && !(flags & BD_GEMM_SINGLE_CTA) && d->sm_count >= 2;
  if (pair) {
    bm = 256;
    m_tiles = (M + bm - 1) / bm;
    tiles = static_cast<int64_t>(m_tiles) * n_tiles;
  }
  const int cta_rows = pair ? 128 : bm;  // token rows loaded per CTA
  const bool use_ws = split_k > 1 && split_mode == BD_SPLIT_REDUCE;
  StreamKSizes sk{0, 0, 0};
  if (streamk) {
    sk = streamk_sizes(M, N, K, d->sm_count);
    if (!workspace || workspace_bytes < sk.total) return BD_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return BD_ERR_ALIGNMENT;
  }
  if (use_ws) {
    const size_t need = static_cast<size_t>(split_k) * M * static_cast<size_t>(N) * sizeof(float);
    if (!workspace || workspace_bytes < need) return BD_ERR_WORKSPACE;
    if (!aligned(workspace, 16) || N % 4) return BD_ERR_ALIGNMENT;
  }

  const int Mp4 = (M + 3) / 4 * 4;
  GemmMaps maps;
  if (!make_map_3d(&maps.a, CU_TENSOR_MAP_DATA_TYPE_UINT8, const_cast<uint8_t*>(a), 128, M, nkt,
                   K, 128, 128, cta_rows, 1, CU_TENSOR_MAP_SWIZZLE_128B))
    return BD_ERR_CUDA;
  if (!make_map_2d(&maps.as, CU_TENSOR_MAP_DATA_TYPE_UINT32, const_cast<uint8_t*>(a_scales), Mp4,
                   nkt, static_cast<uint64_t>(Mp4) * 4, cta_rows, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
    return BD_ERR_CUDA;
  if (!make_map_2d(&maps.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, const_cast<uint8_t*>(b), 64,
                   static_cast<uint64_t>(N) * nkt, 64, 64, 128, CU_TENSOR_MAP_SWIZZLE_64B))
    return BD_ERR_CUDA;
  if (!make_map_2d(&maps.ws, CU_TENSOR_MAP_DATA_TYPE_UINT32, const_cast<uint8_t*>(b_scales), 256,
                   static_cast<uint64_t>(N / 128) * nkt, 1024, 256, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
    return BD_ERR_CUDA;

  GemmParams p;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.tensor_scale = b_tensor_scale;
  p.M = M;
  p.N = N;
  p.K = K;
  p.n_tiles = n_tiles;
  p.m_tiles = m_tiles;
  p.nks = nkt;
  p.n_half_tiles = N / 128;
  p.split_k = streamk ? 0 : split_k;
  p.out_dtype = out_dtype;
  p.epilogue = epilogue;
  p.weights_early = (flags & BD_GEMM_WEIGHTS_STATIC) ? 1 : 0;
  // 128-row tiles, and 64-row tiles with many contributors per tile: partials of 64-128 KB
  // per contributor are summed by a grid of their own (many SMs) instead of by each tile's
  // last contributor (one SM). 64-row tiles with at most ~4 contributors (decode batches of
  // 33-64 tokens on wide N) are summed in-kernel: one launch fewer per GEMM (-2 % at M = 64,
  // N = 14336)
  p.fixup_kernel = (streamk && (bm >= 128 || (bm == 64 && tiles * 4 < d->sm_count))) ? 1 : 0;
  p.vec_out = aligned(c, 16) ? 1 : 0;
  // whole 128-row tiles of a 16-bit C store through shared memory with TMA: boxes of 32 rows x
  // 32 outputs (64 B, the 64B swizzle span), 64 outputs for CTA pairs (128 B, the 128B swizzle
  // span); the row pitch 2N is a multiple of 256 B
  std::memset(&maps.c, 0, sizeof(maps.c));
  p.tma_c = 0;
  if (bm >= 128 && split_mode != BD_SPLIT_ATOMIC && split_k <= 1 && out_dtype != BD_OUT_F32 &&
      p.vec_out) {
    if (!make_map_2d(&maps.c, CU_TENSOR_MAP_DATA_TYPE_UINT16, c, N, M,
                     static_cast<uint64_t>(N) * 2, pair ? 64 : 32, 32,
                     pair ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
      return BD_ERR_CUDA;
    p.tma_c = 1;
  }
  p.err = d->err;
  p.slots = nullptr;
  p.counters = nullptr;
  p.out = c;
  if (split_mode == BD_SPLIT_ATOMIC) p.split_out = kOutAtomic;
  else if (split_k <= 1) p.split_out = kOutC;
  else if (split_mode == BD_SPLIT_REDUCE) {
    p.split_out = kOutPartial;
    p.out = workspace;
  } else p.split_out = kOutPlane;
  const int64_t work = streamk ? tiles * nkt : tiles * split_k;
  if (streamk) {
    p.slots = static_cast<float*>(workspace);
    p.counters = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + sk.slots_bytes);
  }
  // pairs: one cluster of two CTAs per tile in flight, on pairs of SMs
  const int64_t slots = pair ? d->sm_count / 2 : d->sm_count;
  const int grid = static_cast<int>(work < slots ? work : slots) * (pair ? 2 : 1);
  const int rc = launch_gemm_any(bm, (flags & BD_GEMM_B_E4M3) == 0, maps, p, grid,
                                 (flags & BD_GEMM_OVERLAP_PREV) != 0,
                                 as_stream(stream));
  if (rc != BD_OK) return rc;
  if (p.fixup_kernel) return launch_fixup(bm, p, tiles, grid, as_stream(stream));
  if (!use_ws) return rc;
  return bd_splitk_reduce(static_cast<const float*>(workspace), c, bias, b_tensor_scale, M, N,
                          split_k, out_dtype, epilogue, stream);
}

int bd_w4a6_gemm_noalloc(void* c, const uint8_t* a, const uint8_t* a_scales, const uint8_t* b,
                         const uint8_t* b_scales, float b_tensor_scale, const void* bias, int M,
                         int N, int K, int out_dtype, int epilogue, bd_stream_t stream) {
  // the argument checks of bd_w4a6_gemm, before any device call (the scratch clear below)
  if (!c || !a || !a_scales || !b || !b_scales) return BD_ERR_INVALID_ARG;
  if (out_dtype < BD_OUT_BF16 || out_dtype > BD_OUT_F32) return BD_ERR_INVALID_ARG;
  if (epilogue < BD_EPI_NONE || epilogue > BD_EPI_BIAS_GELU) return BD_ERR_INVALID_ARG;
  if (epilogue != BD_EPI_NONE && !bias) return BD_ERR_INVALID_ARG;
  if (M <= 0 || N <= 0 || K <= 0 || N % 128 || K % 128) return BD_ERR_SHAPE;
  if (M > (1 << 30) / 4 || K > (1 << 24) || N > (1 << 24)) return BD_ERR_SHAPE;
  if (!aligned(a, 16) || !aligned(a_scales, 16) || !aligned(b, 16) || !aligned(b_scales, 16) ||
      (bias && !aligned(bias, 2)))
    return BD_ERR_ALIGNMENT;
  DeviceInfo* d = nullptr;
  int st = device_info(&d);
  if (st != BD_OK) return st;
  // the schedule bd_w4a6_gemm picks for split_k = 0: stream-K (needs the scratch) unless the
  // tiles fill the machine twice over
  const int bm = token_tile(M);
  const int64_t tiles =
      static_cast<int64_t>((N + kTileN - 1) / kTileN) * ((M + bm - 1) / bm);
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  if (tiles < 2 * d->sm_count) {
    const StreamKSizes z = streamk_sizes(M, N, K, d->sm_count);
    if (z.total > kNoAllocScratchBytes) return BD_ERR_WORKSPACE;
    st = noalloc_scratch(&scratch);
    if (st != BD_OK) return st;
    // the tile counters must start at zero (a call that ran into a wait limit can leave them
    // set); the slots need no clearing
    if (cudaMemsetAsync(static_cast<uint8_t*>(scratch) + z.slots_bytes, 0, z.counter_bytes,
                        as_stream(stream)) != cudaSuccess)
      return BD_ERR_CUDA;
    scratch_bytes = kNoAllocScratchBytes;
  }
  return bd_w4a6_gemm(c, a, a_scales, b, b_scales, b_tensor_scale, bias, M, N, K, 0,
                      BD_SPLIT_REDUCE, out_dtype, epilogue, scratch, scratch_bytes, stream);
}

}  // extern "C"
