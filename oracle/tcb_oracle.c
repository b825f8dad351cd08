#define _GNU_SOURCE
/*
 * tcb_oracle.c - CPU restatement of TR's quantized-weight matvec path.
 *
 * TEST INFRASTRUCTURE ONLY (see tcb_oracle.h).  Every function names the
 * TR source (path within sekerahmet/TCB) whose arithmetic it restates.
 * Build with -ffp-contract=off: the float operations below must round
 * exactly where TR's Go code rounds; fused steps are written as fmaf().
 */
#include "tcb_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#if defined(__x86_64__)
#include <immintrin.h>
#define TCBO_AVX2 1
#define AVX2_FN __attribute__((target("avx2,fma")))
static int have_avx2(void) {
  static int v = -1;
  if (v < 0) v = __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
  return v;
}
#endif

static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

int tcbo_block_elems(int fmt) {
  switch (fmt) {
  case TCBO_Q8_0: case TCBO_Q4_0: return 32;
  case TCBO_Q4_K: case TCBO_Q6_K: return 256;
  }
  return 0;
}

int tcbo_block_bytes(int fmt) {
  switch (fmt) {
  case TCBO_Q8_0: return 34;
  case TCBO_Q4_0: return 18;
  case TCBO_Q4_K: return 144;
  case TCBO_Q6_K: return 210;
  }
  return 0;
}

/* tensor/cpu_dtype.go:126-145 */
float tcbo_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t ex = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  if (ex == 0x1F) return bits_f(sign | 0x7F800000u | man << 13);
  if (ex == 0) {
    if (man == 0) return bits_f(sign);
    uint32_t e = 127 - 14;
    while ((man & 0x400u) == 0) { man <<= 1; e--; }
    return bits_f(sign | e << 23 | (man & 0x3FFu) << 13);
  }
  return bits_f(sign | (ex + 127 - 15) << 23 | man << 13);
}

/* x86 rule for a NaN result (gpu/kernel_quant.go:13-17, nanRule): the first
 * NaN operand, quieted; with no NaN operand the default NaN 0xFFC00000. */
static inline float nan_rule(float r, float a, float b) {
  if (r == r) return r;
  if (a != a) return bits_f(f_bits(a) | 0x00400000u);
  if (b != b) return bits_f(f_bits(b) | 0x00400000u);
  return bits_f(0xFFC00000u);
}
static inline float mulx(float a, float b) { return nan_rule(a * b, a, b); }
static inline float subx(float a, float b) { return nan_rule(a - b, a, b); }

/* get_scale_min_k4 (tensor/quant.go:158-163) */
static inline void q4k_scale(int j, const uint8_t *q, uint8_t *sc, uint8_t *m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (uint8_t)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

/* tensor/quant.go:139-144 */
static void dq_q8_0(const uint8_t *b, float *y) {
  float d = tcbo_f16_to_f32(rd16(b));
  for (int j = 0; j < 32; j++) y[j] = mulx((float)(int8_t)b[2 + j], d);
}

/* tensor/quant.go:149-155 */
static void dq_q4_0(const uint8_t *b, float *y) {
  float d = tcbo_f16_to_f32(rd16(b));
  for (int j = 0; j < 16; j++) {
    uint8_t q = b[2 + j];
    y[j] = mulx((float)((int)(q & 0xF) - 8), d);
    y[j + 16] = mulx((float)((int)(q >> 4) - 8), d);
  }
}

/* tensor/quant.go:167-182 */
static void dq_q4_k(const uint8_t *b, float *y) {
  float d = tcbo_f16_to_f32(rd16(b)), dmin = tcbo_f16_to_f32(rd16(b + 2));
  const uint8_t *scales = b + 4, *q = b + 16;
  for (int g = 0; g < 4; g++) {
    uint8_t sc, m;
    q4k_scale(2 * g, scales, &sc, &m);
    float d1 = mulx(d, (float)sc), m1 = mulx(dmin, (float)m);
    q4k_scale(2 * g + 1, scales, &sc, &m);
    float d2 = mulx(d, (float)sc), m2 = mulx(dmin, (float)m);
    for (int l = 0; l < 32; l++) {
      y[g * 64 + l] = subx(mulx(d1, (float)(q[l] & 0xF)), m1);
      y[g * 64 + l + 32] = subx(mulx(d2, (float)(q[l] >> 4)), m2);
    }
    q += 32;
  }
}

/* tensor/quant.go:185-204 */
static void dq_q6_k(const uint8_t *b, float *y) {
  const uint8_t *ql = b, *qh = b + 128, *sc = b + 192;
  float d = tcbo_f16_to_f32(rd16(b + 208));
  for (int n = 0; n < 2; n++) {
    float *row = y + n * 128;
    for (int l = 0; l < 32; l++) {
      int is = l / 16;
      uint8_t h = qh[l];
      int q1 = (int)((ql[l] & 0xF) | ((h & 3) << 4)) - 32;
      int q2 = (int)((ql[l + 32] & 0xF) | (((h >> 2) & 3) << 4)) - 32;
      int q3 = (int)((ql[l] >> 4) | (((h >> 4) & 3) << 4)) - 32;
      int q4 = (int)((ql[l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32;
      row[l] = mulx(mulx(d, (float)(int8_t)sc[is]), (float)q1);
      row[l + 32] = mulx(mulx(d, (float)(int8_t)sc[is + 2]), (float)q2);
      row[l + 64] = mulx(mulx(d, (float)(int8_t)sc[is + 4]), (float)q3);
      row[l + 96] = mulx(mulx(d, (float)(int8_t)sc[is + 6]), (float)q4);
    }
    ql += 64;
    qh += 32;
    sc += 8;
  }
}

static void dequant_block(int fmt, const uint8_t *b, float *y) {
  switch (fmt) {
  case TCBO_Q8_0: dq_q8_0(b, y); break;
  case TCBO_Q4_0: dq_q4_0(b, y); break;
  case TCBO_Q4_K: dq_q4_k(b, y); break;
  case TCBO_Q6_K: dq_q6_k(b, y); break;
  }
}

/* tensor/quant.go:207-221 */
void tcbo_dequant(int fmt, const uint8_t *raw, size_t nblocks, float *y) {
  int E = tcbo_block_elems(fmt), B = tcbo_block_bytes(fmt);
  if (!E) return;
  for (size_t i = 0; i < nblocks; i++) dequant_block(fmt, raw + i * B, y + i * E);
}

/* tensor/cpu_gemv.go:66-85 (dot32, Go's unfused x*y then +) */
static float dot32_go(const float *x, const float *y, size_t n) {
  float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t i = 0;
  for (; i + 8 <= n; i += 8)
    for (int j = 0; j < 8; j++) {
      float p = x[i + j] * y[i + j];
      s[j] = s[j] + p;
    }
  for (; i < n; i++) {
    float p = x[i] * y[i];
    s[0] = s[0] + p;
  }
  return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

/* the horizontal reduction of sdot32 (tensor/cpu_gemv_amd64.s:94-104) over
 * lane sums v[j] = (Y0+Y1)+(Y2+Y3) */
static inline float sum32_tree(const float v[8]) {
  float a0 = v[0] + v[4], a1 = v[1] + v[5], a2 = v[2] + v[6], a3 = v[3] + v[7];
  float b0 = a0 + a2, b1 = a1 + a3;
  return b0 + b1;
}

/* tensor/cpu_gemv_amd64.s:65-106 (sdot32): element i goes to accumulator
 * (i/8)%4, lane i%8, with FMA */
static float sdot32_order(const float *x, const float *y, size_t n32) {
  float acc[4][8];
  memset(acc, 0, sizeof acc);
  for (size_t i = 0; i < n32; i += 32)
    for (int a = 0; a < 4; a++)
      for (int l = 0; l < 8; l++)
        acc[a][l] = fmaf(x[i + 8 * a + l], y[i + 8 * a + l], acc[a][l]);
  float v[8];
  for (int l = 0; l < 8; l++) v[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
  return sum32_tree(v);
}

/* tensor/cpu_gemv_amd64.go:25-36 */
float tcbo_dot_f32(const float *x, const float *y, size_t n) {
  if (n < 32) return dot32_go(x, y, n);
  size_t n32 = n & ~(size_t)31;
  float s = sdot32_order(x, y, n32);
  if (n32 < n) s = s + dot32_go(x + n32, y + n32, n - n32);
  return s;
}

#ifdef TCBO_AVX2
/* AVX2 twin of "dequantise + sdot32": same accumulator for every element,
 * same operation order, so the same bits (the property TR's
 * TestQuantDotMatchesOpenedDot asserts for its own kernels). */
AVX2_FN static inline float hsum_acc(__m256 a0, __m256 a1, __m256 a2, __m256 a3) {
  __m256 s = _mm256_add_ps(_mm256_add_ps(a0, a1), _mm256_add_ps(a2, a3));
  float v[8];
  _mm256_storeu_ps(v, s);
  return sum32_tree(v);
}

AVX2_FN static void dq_q4_k_avx2(const uint8_t *b, float *y) {
  float d = tcbo_f16_to_f32(rd16(b)), dmin = tcbo_f16_to_f32(rd16(b + 2));
  const uint8_t *scales = b + 4, *q = b + 16;
  for (int g = 0; g < 4; g++) {
    uint8_t sc, m;
    q4k_scale(2 * g, scales, &sc, &m);
    __m256 d1 = _mm256_set1_ps(d * (float)sc), m1 = _mm256_set1_ps(dmin * (float)m);
    q4k_scale(2 * g + 1, scales, &sc, &m);
    __m256 d2 = _mm256_set1_ps(d * (float)sc), m2 = _mm256_set1_ps(dmin * (float)m);
    for (int l = 0; l < 32; l += 8) {
      __m256i c = _mm256_cvtepu8_epi32(_mm_loadl_epi64((const __m128i *)(q + l)));
      __m256 lo = _mm256_cvtepi32_ps(_mm256_and_si256(c, _mm256_set1_epi32(15)));
      __m256 hi = _mm256_cvtepi32_ps(_mm256_srli_epi32(c, 4));
      /* the product is exact in fp32, so fused and unfused give one rounding */
      _mm256_storeu_ps(y + g * 64 + l, _mm256_fmsub_ps(d1, lo, m1));
      _mm256_storeu_ps(y + g * 64 + l + 32, _mm256_fmsub_ps(d2, hi, m2));
    }
    q += 32;
  }
}

AVX2_FN static void dq_q8_0_avx2(const uint8_t *b, float *y) {
  __m256 d = _mm256_set1_ps(tcbo_f16_to_f32(rd16(b)));
  for (int j = 0; j < 32; j += 8) {
    __m256i c = _mm256_cvtepi8_epi32(_mm_loadl_epi64((const __m128i *)(b + 2 + j)));
    _mm256_storeu_ps(y + j, _mm256_mul_ps(_mm256_cvtepi32_ps(c), d));
  }
}

AVX2_FN static float quant_dot_avx2(int fmt, const float *x, const uint8_t *w, int K) {
  int E = tcbo_block_elems(fmt), B = tcbo_block_bytes(fmt);
  __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
  float buf[256] __attribute__((aligned(32)));
  for (int e0 = 0; e0 < K; e0 += E, w += B) {
    if (fmt == TCBO_Q4_K) dq_q4_k_avx2(w, buf);
    else if (fmt == TCBO_Q8_0) dq_q8_0_avx2(w, buf);
    else dequant_block(fmt, w, buf);
    for (int i = 0; i < E; i += 32) {
      a0 = _mm256_fmadd_ps(_mm256_loadu_ps(x + e0 + i), _mm256_load_ps(buf + i), a0);
      a1 = _mm256_fmadd_ps(_mm256_loadu_ps(x + e0 + i + 8), _mm256_load_ps(buf + i + 8), a1);
      a2 = _mm256_fmadd_ps(_mm256_loadu_ps(x + e0 + i + 16), _mm256_load_ps(buf + i + 16), a2);
      a3 = _mm256_fmadd_ps(_mm256_loadu_ps(x + e0 + i + 24), _mm256_load_ps(buf + i + 24), a3);
    }
  }
  return hsum_acc(a0, a1, a2, a3);
}
#endif

/* tensor/cpu_quant.go:38-44 (dotQuantGo): dequantise then dotF32.  K is a
 * multiple of the block, hence of 32, so dotF32 is sdot32 throughout. */
static float quant_dot_scalar(int fmt, const float *x, const uint8_t *w, int K) {
  int E = tcbo_block_elems(fmt), B = tcbo_block_bytes(fmt);
  float acc[4][8];
  float buf[256];
  memset(acc, 0, sizeof acc);
  for (int e0 = 0; e0 < K; e0 += E, w += B) {
    dequant_block(fmt, w, buf);
    for (int i = 0; i < E; i += 32)
      for (int a = 0; a < 4; a++)
        for (int l = 0; l < 8; l++)
          acc[a][l] = fmaf(x[e0 + i + 8 * a + l], buf[i + 8 * a + l], acc[a][l]);
  }
  float v[8];
  for (int l = 0; l < 8; l++) v[l] = (acc[0][l] + acc[1][l]) + (acc[2][l] + acc[3][l]);
  return sum32_tree(v);
}

float tcbo_quant_dot(int fmt, const float *x, const uint8_t *wrow, int K) {
  if (K <= 0) return 0.0f;
#ifdef TCBO_AVX2
  if (have_avx2()) return quant_dot_avx2(fmt, x, wrow, K);
#endif
  return quant_dot_scalar(fmt, x, wrow, K);
}

/* exported for the AVX2-equals-scalar test */
float tcbo_quant_dot_scalar(int fmt, const float *x, const uint8_t *wrow, int K) {
  if (K <= 0) return 0.0f;
  return quant_dot_scalar(fmt, x, wrow, K);
}

/* ---------------------------------------------------------------------- */
/* row-parallel driver: TR's parallelFor over output rows
 * (tensor/parallel.go:313); each output row is one independent call, so
 * the result does not depend on the split */

typedef void (*row_fn)(void *ctx, int lo, int hi);
typedef struct { row_fn fn; void *ctx; int lo, hi, cpu; } row_job;

/* thread pinning for the timed CPU baseline: worker t runs on the t-th CPU
 * of the process's allowed set (off unless tcbo_set_pinning(1)) */
static int g_pin = 0;
void tcbo_set_pinning(int on) { g_pin = on; }

static int nth_allowed_cpu(int t) {
  cpu_set_t set;
  if (sched_getaffinity(0, sizeof set, &set) != 0) return -1;
  const int n = CPU_COUNT(&set);
  if (n <= 0) return -1;
  int k = t % n;
  for (int c = 0; c < CPU_SETSIZE; c++)
    if (CPU_ISSET(c, &set) && k-- == 0) return c;
  return -1;
}

static void pin_self(int cpu) {
  if (cpu < 0) return;
  cpu_set_t one;
  CPU_ZERO(&one);
  CPU_SET(cpu, &one);
  pthread_setaffinity_np(pthread_self(), sizeof one, &one);
}

static void *row_thread(void *p) {
  row_job *j = (row_job *)p;
  pin_self(j->cpu);
  j->fn(j->ctx, j->lo, j->hi);
  return NULL;
}

static void parallel_rows(int n, int nthreads, row_fn fn, void *ctx) {
  if (nthreads <= 1 || n < 2 * nthreads) {
    fn(ctx, 0, n);
    return;
  }
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  row_job jobs[256];
  int started = 0;
  for (int t = 0; t < nthreads; t++) {
    jobs[t].fn = fn;
    jobs[t].ctx = ctx;
    jobs[t].lo = (int)((long)n * t / nthreads);
    jobs[t].hi = (int)((long)n * (t + 1) / nthreads);
    jobs[t].cpu = g_pin ? nth_allowed_cpu(t) : -1;
    if (t == nthreads - 1) break;
    if (pthread_create(&th[t], NULL, row_thread, &jobs[t]) != 0) break;
    started = t + 1;
  }
  /* this thread takes every slice a worker did not start (on the last
   * slice's CPU when pinned; its own affinity is put back afterwards) */
  cpu_set_t saved;
  const int restore = g_pin && pthread_getaffinity_np(pthread_self(), sizeof saved, &saved) == 0;
  if (g_pin) pin_self(jobs[nthreads - 1].cpu);
  for (int t = started; t < nthreads; t++) fn(ctx, jobs[t].lo, jobs[t].hi);
  if (restore) pthread_setaffinity_np(pthread_self(), sizeof saved, &saved);
  for (int t = 0; t < started; t++) pthread_join(th[t], NULL);
}

typedef struct {
  int fmt, M, N, K;
  const float *a;
  const uint8_t *w;
  float *c;
  size_t rowBytes;
} gemm_ctx;

static void float_rows(void *p, int lo, int hi) {
  gemm_ctx *g = (gemm_ctx *)p;
  for (int m = 0; m < g->M; m++)
    for (int n = lo; n < hi; n++) {
      float v = tcbo_quant_dot(g->fmt, g->a + (size_t)m * g->K, g->w + (size_t)n * g->rowBytes, g->K);
      g->c[(size_t)m * g->N + n] = g->c[(size_t)m * g->N + n] + v;
    }
}

/* tensor/cpu_quant.go:47-160 */
void tcbo_qgemm_float(int fmt, int M, int N, int K, const float *a,
                      const uint8_t *w, float *c, int nthreads) {
  if (K == 0 || M <= 0 || N <= 0 || !tcbo_block_elems(fmt)) return;
  gemm_ctx g = {fmt, M, N, K, a, w, c, (size_t)K / tcbo_block_elems(fmt) * tcbo_block_bytes(fmt)};
  parallel_rows(N, nthreads, float_rows, &g);
}

/* ---------------------------------------------------------------------- */
/* int8-activation path */

/* tensor/cpu_quant_q8.go:39-68 */
void tcbo_quantize_q8(const float *x, int K, int blk, int8_t *q, float *d, int16_t *bs) {
  if (blk != 32 && blk != 256) return;
  for (int b = 0; b < K / blk; b++) {
    const float *v = x + (size_t)b * blk;
    int8_t *qb = q + (size_t)b * blk;
    float amax = 0.0f;
    for (int j = 0; j < blk; j++) {
      float a = fabsf(v[j]);
      if (a > amax) amax = a;
    }
    float id = 127.0f / amax;
    if (!(amax > 0.0f) || (id - id) != 0.0f) {
      memset(qb, 0, (size_t)blk);
      d[b] = 0.0f;
    } else {
      d[b] = amax / 127.0f;
      for (int j = 0; j < blk; j++) {
        float t = v[j] * id;
        double r = nearbyint((double)t); /* round half to even */
        if (r > 127.0) r = 127.0;
        if (r < -127.0) r = -127.0;
        qb[j] = (int8_t)r;
      }
    }
    for (int s = 0; s < blk / 16; s++) {
      int16_t t = 0;
      for (int j = 0; j < 16; j++) t = (int16_t)(t + qb[s * 16 + j]);
      bs[(size_t)b * blk / 16 + s] = t;
    }
  }
}

/* tensor/cpu_quant_q8.go:74-87 */
static float dot_q4_0_q8(int nb, const uint8_t *w, const int8_t *a, const float *d) {
  float acc = 0.0f;
  for (int i = 0; i < nb; i++) {
    const uint8_t *b = w + (size_t)i * 18;
    const int8_t *x = a + (size_t)i * 32;
    int32_t isum = 0;
    for (int j = 0; j < 16; j++)
      isum += ((int32_t)(b[2 + j] & 0xF) - 8) * x[j] + ((int32_t)(b[2 + j] >> 4) - 8) * x[j + 16];
    float t = tcbo_f16_to_f32(rd16(b)) * d[i];
    float p = t * (float)isum;
    acc = acc + p;
  }
  return acc;
}

/* the Q8_0 x Q8 fold, by analogy with dotQ4Q8Go (cpu_quant_q8.go:74-87):
 * isum = sum qw*qx; t = dw*dx; acc += t*isum, each step rounded */
static float dot_q8_0_q8(int nb, const uint8_t *w, const int8_t *a, const float *d) {
  float acc = 0.0f;
  for (int i = 0; i < nb; i++) {
    const uint8_t *b = w + (size_t)i * 34;
    const int8_t *x = a + (size_t)i * 32;
    int32_t isum = 0;
    for (int j = 0; j < 32; j++) isum += (int32_t)(int8_t)b[2 + j] * x[j];
    float t = tcbo_f16_to_f32(rd16(b)) * d[i];
    float p = t * (float)isum;
    acc = acc + p;
  }
  return acc;
}

/* tensor/cpu_quant_q8.go:91-116 */
static float dot_q4_k_q8(int nb, const uint8_t *w, const int8_t *a, const float *d8, const int16_t *bs) {
  float acc = 0.0f;
  for (int i = 0; i < nb; i++) {
    const uint8_t *b = w + (size_t)i * 144;
    float d = tcbo_f16_to_f32(rd16(b)), dmin = tcbo_f16_to_f32(rd16(b + 2));
    const uint8_t *scales = b + 4, *q = b + 16;
    const int8_t *x = a + (size_t)i * 256;
    int32_t isum = 0, msum = 0;
    for (int g = 0; g < 4; g++) {
      uint8_t sc1, m1, sc2, m2;
      q4k_scale(2 * g, scales, &sc1, &m1);
      q4k_scale(2 * g + 1, scales, &sc2, &m2);
      int32_t s1 = 0, s2 = 0;
      for (int l = 0; l < 32; l++) {
        s1 += (int32_t)(q[l] & 0xF) * x[g * 64 + l];
        s2 += (int32_t)(q[l] >> 4) * x[g * 64 + 32 + l];
      }
      isum += (int32_t)sc1 * s1 + (int32_t)sc2 * s2;
      const int16_t *p = bs + (size_t)i * 16 + g * 4;
      msum += (int32_t)m1 * (int32_t)(int16_t)(p[0] + p[1]) + (int32_t)m2 * (int32_t)(int16_t)(p[2] + p[3]);
      q += 32;
    }
    float u = d * (float)isum;
    float v = dmin * (float)msum;
    float t = u - v;
    float p = t * d8[i];
    acc = acc + p;
  }
  return acc;
}

/* tensor/cpu_quant_q8.go:378-407 */
static float dot_q6_k_q8(int nb, const uint8_t *w, const int8_t *a, const float *d8, const int16_t *bs) {
  float acc = 0.0f;
  for (int i = 0; i < nb; i++) {
    const uint8_t *b = w + (size_t)i * 210;
    const uint8_t *ql = b, *qh = b + 128, *sc = b + 192;
    float d = tcbo_f16_to_f32(rd16(b + 208));
    const int8_t *x = a + (size_t)i * 256;
    int32_t isum = 0, msum = 0;
    for (int n = 0; n < 2; n++) {
      for (int l = 0; l < 32; l++) {
        uint8_t h = qh[l];
        int32_t q1 = (int32_t)((ql[l] & 0xF) | ((h & 3) << 4));
        int32_t q2 = (int32_t)((ql[l + 32] & 0xF) | (((h >> 2) & 3) << 4));
        int32_t q3 = (int32_t)((ql[l] >> 4) | (((h >> 4) & 3) << 4));
        int32_t q4 = (int32_t)((ql[l + 32] >> 4) | (((h >> 6) & 3) << 4));
        int is = l / 16;
        isum += (int32_t)(int8_t)sc[is] * q1 * x[n * 128 + l] +
                (int32_t)(int8_t)sc[is + 2] * q2 * x[n * 128 + l + 32] +
                (int32_t)(int8_t)sc[is + 4] * q3 * x[n * 128 + l + 64] +
                (int32_t)(int8_t)sc[is + 6] * q4 * x[n * 128 + l + 96];
      }
      ql += 64;
      qh += 32;
      sc += 8;
    }
    sc = b + 192;
    for (int j = 0; j < 16; j++) msum += (int32_t)(int8_t)sc[j] * (int32_t)bs[(size_t)i * 16 + j];
    float t = d * (float)(isum - 32 * msum);
    float p = t * d8[i];
    acc = acc + p;
  }
  return acc;
}

float tcbo_dot_act8(int fmt, int K, const uint8_t *wrow, const int8_t *q,
                    const float *d, const int16_t *bs) {
  int blk = tcbo_block_elems(fmt);
  if (!blk || K <= 0) return 0.0f;
  int nb = K / blk;
  switch (fmt) {
  case TCBO_Q4_0: return dot_q4_0_q8(nb, wrow, q, d);
  case TCBO_Q8_0: return dot_q8_0_q8(nb, wrow, q, d);
  case TCBO_Q4_K: return dot_q4_k_q8(nb, wrow, q, d, bs);
  case TCBO_Q6_K: return dot_q6_k_q8(nb, wrow, q, d, bs);
  }
  return 0.0f;
}

/* tensor/cpu_quant_q8.go:137-144 */
static int row_finite(const float *a, int K) {
  for (int k = 0; k < K; k++)
    if ((a[k] - a[k]) != 0.0f) return 0;
  return 1;
}

typedef struct {
  gemm_ctx g;
  int blk;
  const int8_t *q;
  const float *d;
  const int16_t *bs;
  const int *rows; /* finite batch rows, quantised in order */
  int nrows;
} act_ctx;

static void act_rows(void *p, int lo, int hi) {
  act_ctx *c = (act_ctx *)p;
  int K = c->g.K, N = c->g.N;
  for (int r = 0; r < c->nrows; r++) {
    int m = c->rows[r];
    const int8_t *q = c->q + (size_t)r * K;
    const float *d = c->d + (size_t)r * (K / c->blk);
    const int16_t *bs = c->bs + (size_t)r * (K / 16);
    for (int n = lo; n < hi; n++) {
      float v = tcbo_dot_act8(c->g.fmt, K, c->g.w + (size_t)n * c->g.rowBytes, q, d, bs);
      c->g.c[(size_t)m * N + n] = c->g.c[(size_t)m * N + n] + v;
    }
  }
}

/* tensor/cpu_quant_q8.go:125-259: a row with a NaN or Inf goes down the
 * float path alone; the other rows are quantised once and dotted with the
 * one-row kernel (multi-row kernels there are bit-identical to it). */
void tcbo_qgemm_act8(int fmt, int M, int N, int K, const float *a,
                     const uint8_t *w, float *c, int nthreads) {
  int blk = tcbo_block_elems(fmt);
  if (K == 0 || M <= 0 || N <= 0 || !blk) return;
  size_t rowBytes = (size_t)K / blk * tcbo_block_bytes(fmt);
  int *rows = (int *)malloc(sizeof(int) * (size_t)M);
  int F = 0;
  for (int m = 0; m < M; m++) {
    if (row_finite(a + (size_t)m * K, K)) {
      rows[F++] = m;
    } else {
      tcbo_qgemm_float(fmt, 1, N, K, a + (size_t)m * K, w, c + (size_t)m * N, nthreads);
    }
  }
  if (F) {
    int8_t *q = (int8_t *)malloc((size_t)F * K);
    float *d = (float *)malloc(sizeof(float) * (size_t)F * (K / blk));
    int16_t *bs = (int16_t *)malloc(sizeof(int16_t) * (size_t)F * (K / 16));
    for (int r = 0; r < F; r++)
      tcbo_quantize_q8(a + (size_t)rows[r] * K, K, blk, q + (size_t)r * K, d + (size_t)r * (K / blk),
                       bs + (size_t)r * (K / 16));
    act_ctx ac = {{fmt, M, N, K, a, w, c, rowBytes}, blk, q, d, bs, rows, F};
    parallel_rows(N, nthreads, act_rows, &ac);
    free(q);
    free(d);
    free(bs);
  }
  free(rows);
}

/* tensor/cpu_quant.go:163-171 */
void tcbo_embedding(int fmt, const uint8_t *raw, int D, const int64_t *idx, int nidx, float *out) {
  int E = tcbo_block_elems(fmt);
  if (!E) return;
  size_t rowBytes = (size_t)D / E * tcbo_block_bytes(fmt);
  for (int i = 0; i < nidx; i++)
    tcbo_dequant(fmt, raw + (size_t)idx[i] * rowBytes, (size_t)D / E, out + (size_t)i * D);
}

/* tensor/quant.go:108-133 */
long tcbo_check_scales(int fmt, const uint8_t *raw, size_t nbytes) {
  int B = tcbo_block_bytes(fmt);
  if (!B) return -1;
  for (size_t b = 0; (b + 1) * B <= nbytes; b++) {
    const uint8_t *p = raw + b * B;
    int bad = 0;
    switch (fmt) {
    case TCBO_Q8_0: case TCBO_Q4_0: bad = (rd16(p) & 0x7C00) == 0x7C00; break;
    case TCBO_Q4_K: bad = (rd16(p) & 0x7C00) == 0x7C00 || (rd16(p + 2) & 0x7C00) == 0x7C00; break;
    case TCBO_Q6_K: bad = (rd16(p + 208) & 0x7C00) == 0x7C00; break;
    }
    if (bad) return (long)b;
  }
  return -1;
}

/* tensor/quant.go:416-427 */
void tcbo_zero_raw(int fmt, uint8_t *raw, size_t nblocks) {
  int B = tcbo_block_bytes(fmt);
  memset(raw, 0, nblocks * (size_t)B);
  if (fmt == TCBO_Q4_0)
    for (size_t b = 0; b < nblocks; b++) memset(raw + b * B + 2, 0x88, (size_t)B - 2);
}

/* tensor/quant_test.go:20-45 */
void tcbo_random_quant(int fmt, uint32_t seed, size_t nblocks, uint8_t *raw) {
  int B = tcbo_block_bytes(fmt);
  uint32_t state = seed;
  for (size_t i = 0; i < nblocks * (size_t)B; i++) {
    state = state * 1664525u + 1013904223u;
    raw[i] = (uint8_t)(state >> 24);
  }
  for (size_t b = 0; b < nblocks; b++) {
    uint8_t *p = raw + b * B;
    int at[2] = {-1, -1};
    switch (fmt) {
    case TCBO_Q8_0: case TCBO_Q4_0: at[0] = 0; break;
    case TCBO_Q4_K: at[0] = 0; at[1] = 2; break;
    case TCBO_Q6_K: at[0] = 208; break;
    }
    for (int k = 0; k < 2; k++) {
      if (at[k] < 0) continue;
      uint16_t v = rd16(p + at[k]);
      if ((v & 0x7C00) == 0x7C00) {
        v = (uint16_t)(v & ~0x4000);
        p[at[k]] = (uint8_t)v;
        p[at[k] + 1] = (uint8_t)(v >> 8);
      }
    }
  }
}

uint64_t tcbo_fnv1a_f32(const float *y, size_t n) {
  uint64_t h = 14695981039346656037ull;
  for (size_t i = 0; i < n; i++) {
    uint32_t u = f_bits(y[i]);
    for (int k = 0; k < 4; k++) {
      h ^= (uint8_t)(u >> (8 * k));
      h *= 1099511628211ull;
    }
  }
  return h;
}
