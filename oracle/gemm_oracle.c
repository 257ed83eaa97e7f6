/* gemm_oracle.c — CPU oracle for the B200 GEMM path. TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the reference's host-side arithmetic for the
 * GEMM experiments so that tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs can check and time the CUDA path. Nothing
 * in the product library links or calls it.
 *
 * What it restates (reference = TheManWhoIsStupid/Hopper-lab):
 *   - make_random_vector (include/common/tensor.h:12-20): std::mt19937 seeded with
 *     `seed`, std::uniform_real_distribution<float>(lo, hi). The libstdc++ forms
 *     of both are restated: MT19937 from Matsumoto & Nishimura (1998) with the
 *     C++11 seeding recurrence, and generate_canonical<float, 24> (one 32-bit draw,
 *     u / 2^32 in float, clamped below 1) followed by u * (hi - lo) + lo.
 *   - std::normal_distribution<float> (Marsaglia polar method, libstdc++ form),
 *     used by the bf16 config's normal(0,1)*0.1 inputs.
 *   - the fp16 / bf16 / e4m3 casts the experiments apply to those floats
 *     (src/05_gemm/gemm_ws.cu:249, src/07_fp8/gemm_fp8.cu:182-186): IEEE
 *     round-to-nearest-even; e4m3 saturates to ±448 (SATFINITE), as the
 *     __nv_fp8_e4m3(float) constructor does.
 *   - the host reference GEMM (src/05_gemm/gemm_ws.cu:258-265,
 *     src/07_fp8/gemm_fp8.cu:246-253): acc = 0.f; acc += float(a[m*K+k]) *
 *     float(b[n*K+k]) for k = 0..K-1, in fp32, sequential in k. Compiled with
 *     -ffp-contract=off so the product and the sum round separately, as the
 *     reference's host compiler does on x86-64.
 *   - check_close (include/common/checker.h:30-55): count of
 *     |g - e| > atol + rtol*|e|, max abs and max rel error.
 *
 * Pinned against the reference's own code: oracle/_ref compiles the reference's
 * include/common/tensor.h and checker.h plus the CUDA headers' conversions, and
 * tests/golden holds fixtures generated from it (tests/golden/make_golden.py).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------- MT19937 ------------------------------------ */
typedef struct {
  uint32_t x[624];
  int i;
} mt_t;

static void mt_seed(mt_t* s, uint32_t seed) {
  s->x[0] = seed;
  for (int i = 1; i < 624; ++i) s->x[i] = 1812433253u * (s->x[i - 1] ^ (s->x[i - 1] >> 30)) + (uint32_t)i;
  s->i = 624;
}

static void mt_twist(mt_t* s) {
  for (int i = 0; i < 624; ++i) {
    const uint32_t y = (s->x[i] & 0x80000000u) | (s->x[(i + 1) % 624] & 0x7fffffffu);
    uint32_t v = s->x[(i + 397) % 624] ^ (y >> 1);
    if (y & 1u) v ^= 0x9908b0dfu;
    s->x[i] = v;
  }
  s->i = 0;
}

static uint32_t mt_next(mt_t* s) {
  if (s->i >= 624) mt_twist(s);
  uint32_t y = s->x[s->i++];
  y ^= y >> 11;
  y ^= (y << 7) & 0x9d2c5680u;
  y ^= (y << 15) & 0xefc60000u;
  y ^= y >> 18;
  return y;
}

/* generate_canonical<float, 24> over a 32-bit engine: a single draw. */
static float canonical_f(mt_t* s) {
  volatile float sum = (float)mt_next(s);
  volatile float r = 4294967296.0f;
  float ret = sum / r;
  if (ret >= 1.0f) ret = nextafterf(1.0f, 0.0f);
  return ret;
}

void oracle_uniform(uint32_t seed, int64_t n, float lo, float hi, float* out) {
  mt_t s;
  mt_seed(&s, seed);
  const float span = hi - lo;
  for (int64_t i = 0; i < n; ++i) {
    volatile float t = canonical_f(&s) * span;
    out[i] = t + lo;
  }
}

void oracle_normal(uint32_t seed, int64_t n, float mean, float stddev, float* out) {
  mt_t s;
  mt_seed(&s, seed);
  int have = 0;
  float saved = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    float ret;
    if (have) {
      have = 0;
      ret = saved;
    } else {
      float x, y, r2;
      do {
        volatile float cx = 2.0f * canonical_f(&s);
        x = cx - 1.0f;
        volatile float cy = 2.0f * canonical_f(&s);
        y = cy - 1.0f;
        volatile float xx = x * x, yy = y * y;
        r2 = xx + yy;
      } while (r2 > 1.0f || r2 == 0.0f);
      volatile float lg = -2.0f * logf(r2);
      volatile float q = lg / r2;
      const float mult = sqrtf(q);
      volatile float sx = x * mult;
      saved = sx;
      have = 1;
      ret = y * mult;
    }
    volatile float t = ret * stddev;
    out[i] = t + mean;
  }
}

/* --------------------------- narrow float formats --------------------------- */
static uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* Generic IEEE-style encoder: round-to-nearest-even of a finite float to a format
 * with `mbits` mantissa bits, exponent bias `bias`, and largest finite magnitude
 * `maxf`. Returns sign|magnitude bits; `sat` saturates to maxf, else overflow -> inf
 * code `inf_code` (or NaN code when the format has no infinity). */
static uint32_t encode_small(float f, int mbits, int bias, int min_exp, float maxf, uint32_t max_code,
                             uint32_t inf_code, uint32_t nan_code, int sign_shift, int sat) {
  const uint32_t u = f2u(f);
  const uint32_t sign = (u >> 31) << sign_shift;
  if ((u & 0x7fffffffu) > 0x7f800000u) return nan_code; /* canonical (positive) NaN */
  const float a = fabsf(f);
  if (isinf(a)) return sat ? (sign | max_code) : (sign | inf_code);
  if (a == 0.0f) return sign;
  /* Exact RNE via scaled integer rounding in double. */
  int e;
  frexp((double)a, &e); /* a = m * 2^e, m in [0.5, 1) */
  int exp_unb = e - 1;  /* a in [2^exp_unb, 2^(exp_unb+1)) */
  if (exp_unb < min_exp) exp_unb = min_exp; /* subnormal range: fixed quantum */
  const double quantum = ldexp(1.0, exp_unb - mbits);
  double q = (double)a / quantum; /* exact: a has 24 bits, quantum power of 2 */
  double fl = floor(q);
  double rem = q - fl;
  double r = fl;
  if (rem > 0.5 || (rem == 0.5 && fmod(fl, 2.0) != 0.0)) r = fl + 1.0;
  double val = r * quantum;
  if (val > (double)maxf) {
    /* overflow beyond the largest finite value after rounding */
    return sat ? (sign | max_code) : (sign | inf_code);
  }
  if (val == 0.0) return sign;
  /* re-encode val */
  int e2;
  frexp(val, &e2);
  int ue = e2 - 1;
  uint32_t code;
  if (ue < min_exp) { /* subnormal */
    code = (uint32_t)(val / ldexp(1.0, min_exp - mbits));
  } else {
    const uint32_t mant = (uint32_t)((val / ldexp(1.0, ue) - 1.0) * ldexp(1.0, mbits) + 0.5);
    code = ((uint32_t)(ue + bias) << mbits) | mant;
  }
  return sign | code;
}

uint16_t oracle_f32_to_f16_1(float f) {
  /* binary16: 10 mantissa bits, bias 15, min normal exponent -14, max 65504, inf 0x7c00 */
  return (uint16_t)encode_small(f, 10, 15, -14, 65504.0f, 0x7bffu, 0x7c00u, 0x7fffu, 15, 0);
}

float oracle_f16_to_f32_1(uint16_t h) {
  const uint32_t s = (uint32_t)(h >> 15) & 1u, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  float v;
  if (e == 0) v = ldexpf((float)m, -24);
  else if (e == 31 && m) return u2f(0x7fffffffu); /* canonical NaN, as the CUDA header */
  else if (e == 31) v = INFINITY;
  else v = ldexpf((float)(m | 0x400u), (int)e - 25);
  return s ? -v : v;
}

uint16_t oracle_f32_to_bf16_1(float f) {
  const uint32_t u = f2u(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fffu; /* canonical NaN, as the CUDA header */
  const uint32_t lsb = (u >> 16) & 1u;
  return (uint16_t)((u + 0x7fffu + lsb) >> 16);
}

float oracle_bf16_to_f32_1(uint16_t b) { return u2f((uint32_t)b << 16); }

uint8_t oracle_f32_to_e4m3_1(float f) {
  /* OCP e4m3 ("fn"): 3 mantissa bits, bias 7, min normal exponent -6, max 448,
   * no infinity, NaN = S.1111.111. SATFINITE: overflow and inf clamp to ±448. */
  return (uint8_t)encode_small(f, 3, 7, -6, 448.0f, 0x7eu, 0x7eu, 0x7fu, 7, 1);
}

float oracle_e4m3_to_f32_1(uint8_t q) {
  const uint32_t s = (q >> 7) & 1u, e = (q >> 3) & 0xfu, m = q & 0x7u;
  float v;
  if (e == 15 && m == 7) return u2f(0x7fffffffu); /* canonical NaN, as the CUDA header */
  else if (e == 0) v = ldexpf((float)m, -9);
  else v = ldexpf((float)(m | 0x8u), (int)e - 10);
  return s ? -v : v;
}

void oracle_f32_to_f16(const float* x, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f32_to_f16_1(x[i]);
}
void oracle_f16_to_f32(const uint16_t* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f16_to_f32_1(x[i]);
}
void oracle_f32_to_bf16(const float* x, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f32_to_bf16_1(x[i]);
}
void oracle_bf16_to_f32(const uint16_t* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_bf16_to_f32_1(x[i]);
}
void oracle_f32_to_e4m3(const float* x, int64_t n, uint8_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_f32_to_e4m3_1(x[i]);
}
void oracle_e4m3_to_f32(const uint8_t* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_e4m3_to_f32_1(x[i]);
}

/* Per-tensor scaled quantisation of the build's fp8 configs: scale = amax/448
 * (1 when amax == 0), q = e4m3(x / scale). Returns the scale. */
float oracle_quantize_e4m3_scaled(const float* x, int64_t n, uint8_t* q) {
  float amax = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    const float a = fabsf(x[i]);
    if (a > amax) amax = a;
  }
  const float scale = amax > 0.0f ? amax / 448.0f : 1.0f;
  for (int64_t i = 0; i < n; ++i) q[i] = oracle_f32_to_e4m3_1(x[i] / scale);
  return scale;
}

/* ------------------------------- reference GEMM ----------------------------- */
typedef struct {
  const float* A;
  const float* B;
  const float* Bt; /* K x N transposed copy (blocked variant) */
  float* C;
  int64_t M, N, K, ldc;
  int64_t r0, r1;
  int naive;
  int64_t next; /* row counter (shared) */
  pthread_mutex_t* mu;
} gemm_job_t;

/* The reference's loop, verbatim order: for m, for n, for k. */
static void gemm_rows_naive(const float* A, const float* B, float* C, int64_t N, int64_t K,
                            int64_t ldc, int64_t m) {
  const float* a = A + m * K;
  for (int64_t n = 0; n < N; ++n) {
    const float* b = B + n * K;
    float acc = 0.0f;
    for (int64_t k = 0; k < K; ++k) acc += a[k] * b[k];
    C[m * ldc + n] = acc;
  }
}

/* Same arithmetic per output element (fp32, sequential in k, product and sum
 * rounded separately), evaluated for 64 columns at a time over a transposed B so
 * the compiler can run independent columns in SIMD lanes. Bit-identical to the
 * naive order; tests check that. */
static void gemm_rows_blocked(const float* A, const float* Bt, float* C, int64_t N, int64_t K,
                              int64_t ldc, int64_t m) {
  const float* a = A + m * K;
  enum { NB = 64 };
  for (int64_t n0 = 0; n0 < N; n0 += NB) {
    const int64_t nb = (N - n0) < NB ? (N - n0) : NB;
    float acc[NB];
    for (int j = 0; j < NB; ++j) acc[j] = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
      const float av = a[k];
      const float* brow = Bt + k * N + n0;
      if (nb == NB) {
        for (int j = 0; j < NB; ++j) acc[j] += av * brow[j];
      } else {
        for (int64_t j = 0; j < nb; ++j) acc[j] += av * brow[j];
      }
    }
    for (int64_t j = 0; j < nb; ++j) C[m * ldc + n0 + j] = acc[j];
  }
}

static void* gemm_worker(void* p) {
  gemm_job_t* j = (gemm_job_t*)p;
  for (;;) {
    pthread_mutex_lock(j->mu);
    const int64_t m = j->next++;
    pthread_mutex_unlock(j->mu);
    if (m >= j->r1) break;
    if (j->naive) gemm_rows_naive(j->A, j->B, j->C, j->N, j->K, j->ldc, m);
    else gemm_rows_blocked(j->A, j->Bt, j->C, j->N, j->K, j->ldc, m);
  }
  return NULL;
}

/* C[r0:r1, :] (row-major, leading dim ldc, rows indexed absolutely) =
 * A[r0:r1, :] . B^T, A M x K, B N x K, both row-major fp32. naive != 0 keeps the
 * reference's m-n-k order; otherwise the bit-identical blocked form is used.
 * threads <= 0 selects 1. */
int oracle_gemm_tn(const float* A, const float* B, int64_t M, int64_t N, int64_t K, int64_t r0,
                   int64_t r1, float* C, int64_t ldc, int threads, int naive) {
  if (r0 < 0 || r1 > M || r0 > r1) return -1;
  if (threads <= 0) threads = 1;
  float* Bt = NULL;
  if (!naive) {
    Bt = (float*)malloc((size_t)(N * K) * sizeof(float));
    if (!Bt) return -2;
    for (int64_t n = 0; n < N; ++n)
      for (int64_t k = 0; k < K; ++k) Bt[k * N + n] = B[n * K + k];
  }
  pthread_mutex_t mu;
  pthread_mutex_init(&mu, NULL);
  gemm_job_t job = {A, B, Bt, C, M, N, K, ldc, r0, r1, naive, r0, &mu};
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
  for (int t = 0; t < threads; ++t) pthread_create(&th[t], NULL, gemm_worker, &job);
  for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
  free(th);
  pthread_mutex_destroy(&mu);
  free(Bt);
  return 0;
}

/* ------------------------------- check_close -------------------------------- */
typedef struct {
  int64_t n;
  int64_t mismatches;
  double max_abs_err;
  double max_rel_err;
} oracle_report_t;

int oracle_check_close(const float* got, const float* ref, int64_t n, double rtol, double atol,
                       oracle_report_t* r) {
  r->n = n;
  r->mismatches = 0;
  r->max_abs_err = 0.0;
  r->max_rel_err = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    const double g = (double)got[i], e = (double)ref[i];
    const double diff = fabs(g - e);
    const double rel = diff / fmax(fabs(e), 1e-30);
    if (diff > r->max_abs_err) r->max_abs_err = diff;
    if (rel > r->max_rel_err) r->max_rel_err = rel;
    if (diff > atol + rtol * fabs(e)) ++r->mismatches;
  }
  return r->mismatches == 0;
}
