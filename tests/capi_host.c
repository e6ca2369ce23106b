/* A plain C host of the library's C ABI (include/bitdance_b200.h), as a non-Python caller binds
 * it: links libbitdance_b200.so and makes the calls that need no GPU -- version, status text,
 * workspace sizing and the argument checks every entry point performs before it touches a
 * device. Built and run by tests/test_capi_c.py; prints "ok" and exits 0 when every check holds. */
#include <stdint.h>
#include <stdio.h>

#include "bitdance_b200.h"

static int fails = 0;

static void expect(const char* what, long got, long want) {
  if (got != want) {
    printf("FAIL %s: got %ld, want %ld\n", what, got, want);
    ++fails;
  }
}

int main(void) {
  /* never dereferenced: every call below fails its argument checks first */
  void* ok = (void*)(uintptr_t)4096;
  uint8_t* u8 = (uint8_t*)ok;
  uint8_t* odd = (uint8_t*)(uintptr_t)4097;

  expect("version", bd_version() >= 100, 1);
  printf("status text of BD_ERR_SHAPE: %s\n", bd_status_string(BD_ERR_SHAPE));

  expect("split-K workspace bytes", (long)bd_query_workspace(64, 1024, 1024, 4, BD_SPLIT_REDUCE),
         4L * 64 * 1024 * 4);
  expect("no workspace for split_k = 1", (long)bd_query_workspace(64, 1024, 1024, 1, BD_SPLIT_REDUCE),
         0);
  expect("workspace of an unsupported shape", (long)bd_query_workspace(64, 1000, 1024, 4, 0), 0);

  expect("gemm: null output",
         bd_w4a6_gemm(NULL, u8, u8, u8, u8, 1.0f, NULL, 16, 128, 128, 1, BD_SPLIT_REDUCE,
                      BD_OUT_BF16, BD_EPI_NONE, NULL, 0, NULL),
         BD_ERR_INVALID_ARG);
  expect("gemm: N % 128",
         bd_w4a6_gemm(ok, u8, u8, u8, u8, 1.0f, NULL, 16, 100, 128, 1, BD_SPLIT_REDUCE,
                      BD_OUT_BF16, BD_EPI_NONE, NULL, 0, NULL),
         BD_ERR_SHAPE);
  expect("gemm: misaligned A",
         bd_w4a6_gemm(ok, odd, u8, u8, u8, 1.0f, NULL, 16, 128, 128, 1, BD_SPLIT_REDUCE,
                      BD_OUT_BF16, BD_EPI_NONE, NULL, 0, NULL),
         BD_ERR_ALIGNMENT);
  expect("gemm_ex: unknown flag",
         bd_w4a6_gemm_ex(ok, u8, u8, u8, u8, 1.0f, NULL, 16, 128, 128, 1, BD_SPLIT_REDUCE,
                         BD_OUT_BF16, BD_EPI_NONE, NULL, 0, 16u, NULL),
         BD_ERR_INVALID_ARG);
  expect("noalloc: bias epilogue without bias",
         bd_w4a6_gemm_noalloc(ok, u8, u8, u8, u8, 1.0f, NULL, 16, 128, 128, BD_OUT_BF16,
                              BD_EPI_BIAS, NULL),
         BD_ERR_INVALID_ARG);
  expect("transcode: scale block 24",
         bd_transcode_nvfp4_to_mxfp6(u8, u8, u8, u8, 8, 24, NULL), BD_ERR_INVALID_ARG);
  expect("transcode: empty input", bd_transcode_nvfp4_to_mxfp6(u8, u8, u8, u8, 0, 16, NULL),
         BD_OK);
  expect("pack_b: K % 128", bd_pack_b(u8, u8, u8, u8, 128, 100, NULL), BD_ERR_SHAPE);
  expect("pack_a: K % 128", bd_pack_a(u8, u8, u8, u8, 4, 100, NULL), BD_ERR_SHAPE);
  expect("splitk_reduce: N % 4",
         bd_splitk_reduce((const float*)ok, ok, NULL, 1.0f, 4, 6, 2, BD_OUT_BF16, BD_EPI_NONE,
                          NULL),
         BD_ERR_SHAPE);
  expect("quantize A: K % 32",
         bd_quantize_a_mxfp6(ok, BD_IN_BF16, u8, u8, NULL, 4, 48, NULL), BD_ERR_SHAPE);
  expect("quantize A ex: unknown flag",
         bd_quantize_a_mxfp6_ex(ok, BD_IN_F32, u8, u8, NULL, 4, 128, 2u, NULL),
         BD_ERR_INVALID_ARG);
  expect("quantize B: K % 16",
         bd_quantize_b_nvfp4(ok, BD_IN_F32, u8, u8, (uint32_t*)ok, 4, 40, NULL), BD_ERR_SHAPE);
  expect("self-test: limit too small", bd_selftest_bounded_wait(10, NULL), BD_ERR_INVALID_ARG);
  expect("device_error: null word", bd_device_error(NULL, 0), BD_ERR_INVALID_ARG);

  if (fails == 0) printf("ok\n");
  return fails != 0;
}
