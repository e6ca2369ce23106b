/*
 * w4a6_ref.c -- CPU restatement of the NVFP4 -> MXFP6 transcode and of the MXFP6
 * dequantisation. TEST INFRASTRUCTURE ONLY: it is the checker for the CUDA path and the
 * timed CPU baseline; the product library never links or calls it.
 *
 * It follows the reference project's algorithm (paths inside scimg/bitdance):
 *   - E4M3 byte decode with renormalised subnormals:   kernel/transcode_lut.py:61-76
 *   - CODE_LUT / BUMP_LUT derivation (nearest E2M3 magnitude, ties to the lower
 *     magnitude because argmin keeps the first minimum): kernel/transcode_lut.py:79-96,
 *     vector_quant_error.py:255-280
 *   - per-32 transcode  e8m0 = exp + bump + 127, e2m3 = sign<<5 | CODE_LUT[mb][mag]:
 *     kernel/nvfp4_codec.py:66-76
 *   - dequantisation:   kernel/nvfp4_codec.py:79-85
 * and adds the per-16 pair rule (two E4M3 16-blocks -> one E8M0 32-block; each half folds
 * its own mantissa and its relative exponent d = emax - (exp + bump), clamped at 7 where
 * every product rounds to zero).
 *
 * Packed NVFP4 input: element 2j in the low nibble of byte j, element 2j+1 in the high.
 * Output E2M3 codes: one code per byte, code in bits [5:0].
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

static const double kE2M1[8] = {0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0};
static const int kSubMant[8] = {0, 0, 0, 4, 0, 2, 4, 6};    /* transcode_lut.py:61 */
static const int kSubExp[8] = {0, -9, -8, -8, -7, -7, -7, -7}; /* transcode_lut.py:62 */

static double e2m3_mag(int i) { /* vector_quant_error.py:42-51 */
  int e = i >> 3, m = i & 7;
  return e == 0 ? m / 8.0 : (1.0 + m / 8.0) * ldexp(1.0, e - 1);
}

/* nearest E2M3 magnitude index, first minimum wins (ties -> lower magnitude) */
static int nearest_e2m3(double x) {
  int best = 0;
  double bd = fabs(x - e2m3_mag(0));
  for (int i = 1; i < 32; ++i) {
    double d = fabs(x - e2m3_mag(i));
    if (d < bd) { bd = d; best = i; }
  }
  return best;
}


/* ---- static-partition parallel-for over pthreads (no OpenMP runtime in this image) ---- */
typedef void (*range_fn)(const void* ctx, int64_t lo, int64_t hi);
typedef struct { range_fn fn; const void* ctx; int64_t lo, hi; } range_job;

static void* range_thread(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->ctx, j->lo, j->hi);
  return NULL;
}

static void parallel_for(int64_t n, int nthreads, range_fn fn, const void* ctx) {
  enum { kMaxThreads = 256 };
  if (nthreads > kMaxThreads) nthreads = kMaxThreads;
  if (nthreads <= 1 || n < 4096) { fn(ctx, 0, n); return; }
  pthread_t th[kMaxThreads];
  range_job jobs[kMaxThreads];
  int created[kMaxThreads];
  int64_t chunk = (n + nthreads - 1) / nthreads;
  for (int t = 0; t < nthreads; ++t) {
    int64_t lo = (int64_t)t * chunk, hi = lo + chunk < n ? lo + chunk : n;
    created[t] = 0;
    if (lo >= hi) continue;
    jobs[t].fn = fn; jobs[t].ctx = ctx; jobs[t].lo = lo; jobs[t].hi = hi;
    if (pthread_create(&th[t], NULL, range_thread, &jobs[t]) == 0) created[t] = 1;
    else fn(ctx, lo, hi);
  }
  for (int t = 0; t < nthreads; ++t)
    if (created[t]) pthread_join(th[t], NULL);
}

static uint8_t g_code[64], g_bump[8], g_pair[512];
static int g_ready = 0;

static void build_tables(void) {
  if (g_ready) return;
  for (int mb = 0; mb < 8; ++mb) {
    double m = 1.0 + mb / 8.0;
    int bump = m > 1.0 ? 1 : 0;
    g_bump[mb] = (uint8_t)bump;
    for (int d = 0; d < 8; ++d)
      for (int g = 0; g < 8; ++g) {
        int c = nearest_e2m3(m * kE2M1[g] / ldexp(1.0, bump + d));
        g_pair[(mb * 8 + d) * 8 + g] = (uint8_t)c;
        if (d == 0) g_code[mb * 8 + g] = (uint8_t)c;
      }
  }
  g_ready = 1;
}

/* Copy out the tables: code_lut[64] (mb*8+mag), bump_lut[8], pair_lut[512] ((mb*8+d)*8+mag). */
void orc_tables(uint8_t* code_lut, uint8_t* bump_lut, uint8_t* pair_lut) {
  build_tables();
  if (code_lut) memcpy(code_lut, g_code, 64);
  if (bump_lut) memcpy(bump_lut, g_bump, 8);
  if (pair_lut) memcpy(pair_lut, g_pair, 512);
}

static inline void decode_e4m3(int byte, int* mb, int* exp) {
  int eb = (byte >> 3) & 0xF, k = byte & 7;
  if (eb == 0) { *mb = kSubMant[k]; *exp = kSubExp[k]; }
  else { *mb = k; *exp = eb - 7; }
}

static void transcode_block(const uint8_t* packed16, const uint8_t* sc, int scale_block,
                            uint8_t* out32, uint8_t* e8) {
  int mb[2], ex[2], e[2];
  decode_e4m3(sc[0], &mb[0], &ex[0]);
  if (scale_block == 16) decode_e4m3(sc[1], &mb[1], &ex[1]);
  else { mb[1] = mb[0]; ex[1] = ex[0]; }
  e[0] = ex[0] + g_bump[mb[0]];
  e[1] = ex[1] + g_bump[mb[1]];
  int emax = e[0] > e[1] ? e[0] : e[1];
  *e8 = (uint8_t)(emax + 127);
  for (int h = 0; h < 2; ++h) {
    int d = emax - e[h];
    if (d > 7) d = 7;
    const uint8_t* lut = &g_pair[(mb[h] * 8 + d) * 8];
    for (int i = 0; i < 16; ++i) {
      int idx = h * 16 + i;
      int nib = (packed16[idx >> 1] >> ((idx & 1) * 4)) & 0xF;
      out32[idx] = (uint8_t)(((nib >> 3) << 5) | lut[nib & 7]);
    }
  }
}

typedef struct {
  const uint8_t* codes; const uint8_t* scales; int scale_block; uint8_t* e2m3; uint8_t* e8m0;
} transcode_ctx;

static void transcode_range(const void* p, int64_t lo, int64_t hi) {
  const transcode_ctx* c = (const transcode_ctx*)p;
  const int spb = c->scale_block == 16 ? 2 : 1;
  for (int64_t b = lo; b < hi; ++b)
    transcode_block(c->codes + b * 16, c->scales + b * spb, c->scale_block, c->e2m3 + b * 32,
                    c->e8m0 + b);
}

/* nblk32 blocks of 32 codes. codes_packed: 16 B/block. scales: 2 B/block (scale_block 16)
 * or 1 B/block (32). e2m3: 32 B/block. e8m0: 1 B/block. Returns 0, or -1 on bad args. */
int orc_transcode(const uint8_t* codes_packed, const uint8_t* scales, int64_t nblk32,
                  int scale_block, uint8_t* e2m3, uint8_t* e8m0, int nthreads) {
  if (scale_block != 16 && scale_block != 32) return -1;
  if (nblk32 < 0) return -1;
  build_tables();
  transcode_ctx c = {codes_packed, scales, scale_block, e2m3, e8m0};
  parallel_for(nblk32, nthreads, transcode_range, &c);
  return 0;
}

typedef struct { const uint8_t* e2m3; const uint8_t* e8m0; float* out; float val[64]; } dequant_ctx;

static void dequant_range(const void* p, int64_t lo, int64_t hi) {
  const dequant_ctx* c = (const dequant_ctx*)p;
  for (int64_t b = lo; b < hi; ++b) {
    const float s = ldexpf(1.0f, (int)c->e8m0[b] - 127);
    const uint8_t* in = c->e2m3 + b * 32;
    float* out = c->out + b * 32;
    for (int i = 0; i < 32; ++i) out[i] = c->val[in[i] & 63] * s;
  }
}

/* MXFP6 -> float: out[b*32+i] = (+-)E2M3(e2m3) * 2^(e8m0-127) (kernel/nvfp4_codec.py:79-85). */
int orc_dequant(const uint8_t* e2m3, const uint8_t* e8m0, int64_t nblk32, float* out,
                int nthreads) {
  if (nblk32 < 0) return -1;
  dequant_ctx c;
  c.e2m3 = e2m3; c.e8m0 = e8m0; c.out = out;
  for (int i = 0; i < 64; ++i) c.val[i] = (i & 32 ? -1.0f : 1.0f) * (float)e2m3_mag(i & 31);
  parallel_for(nblk32, nthreads, dequant_range, &c);
  return 0;
}
