/*
 * oracle/mcke_oracle.c -- CPU restatement of mini-cuda-kernel-engine's CPU
 * oracle (tests/reference.hpp).  TEST INFRASTRUCTURE ONLY: see mcke_oracle.h.
 *
 * Built with -ffp-contract=off so that no multiply-add is fused: the reference
 * is plain IEEE double arithmetic and the restatement must round the same way.
 */
#include "mcke_oracle.h"

#include <math.h>
#include <string.h>

/* ---------------------------------------------------------------------------
 * mt19937_64.  The published 64-bit Mersenne Twister (Nishimura 2000), with the
 * parameter set the C++ standard specifies for std::mt19937_64
 * ([rand.predef]: w=64 n=312 m=156 r=31 a=0xb5026f5aa96619e9 u=29
 * d=0x5555555555555555 s=17 b=0x71d67fffeda60000 t=37 c=0xfff7eee000000000
 * l=43 f=6364136223846793005).  The reference draws all of its test data from
 * this engine (tests/reference.hpp:103, :407).
 * ------------------------------------------------------------------------- */
#define MT_N 312
#define MT_M 156
#define MT_UPPER 0xFFFFFFFF80000000ULL
#define MT_LOWER 0x000000007FFFFFFFULL

void oracle_mt64_seed(oracle_mt64* e, uint64_t seed) {
  e->mt[0] = seed;
  for (int i = 1; i < MT_N; ++i)
    e->mt[i] = 6364136223846793005ULL * (e->mt[i - 1] ^ (e->mt[i - 1] >> 62)) + (uint64_t)i;
  e->idx = MT_N;
}

static void mt64_twist(oracle_mt64* e) {
  for (int i = 0; i < MT_N; ++i) {
    const uint64_t y = (e->mt[i] & MT_UPPER) | (e->mt[(i + 1) % MT_N] & MT_LOWER);
    uint64_t v = e->mt[(i + MT_M) % MT_N] ^ (y >> 1);
    if (y & 1ULL) v ^= 0xB5026F5AA96619E9ULL;
    e->mt[i] = v;
  }
  e->idx = 0;
}

uint64_t oracle_mt64_next(oracle_mt64* e) {
  if (e->idx >= MT_N) mt64_twist(e);
  uint64_t x = e->mt[e->idx++];
  x ^= (x >> 29) & 0x5555555555555555ULL;
  x ^= (x << 17) & 0x71D67FFFEDA60000ULL;
  x ^= (x << 37) & 0xFFF7EEE000000000ULL;
  x ^= (x >> 43);
  return x;
}

/* tests/reference.hpp:101-109.  The top 24 bits of each draw, scaled into
 * [lo, hi] in double, stored as float.  `hi - lo` is a float subtraction in the
 * reference (both operands are float), kept as one here. */
void oracle_fill_random(float* p, size_t n, uint64_t seed, float lo, float hi) {
  oracle_mt64 e;
  oracle_mt64_seed(&e, seed);
  const float span = hi - lo;
  for (size_t i = 0; i < n; ++i) {
    const double u = (double)(oracle_mt64_next(&e) >> 40) / (double)(1u << 24);
    p[i] = (float)((double)lo + u * (double)span);
  }
}

/* Not in the reference (it has no normal generator).  Builder convention:
 * Box-Muller over pairs of the same 24-bit uniforms fill_random uses,
 * z0 = sqrt(-2 ln(1-u1)) cos(2 pi u2), z1 = ... sin(...), written in order. */
void oracle_fill_normal(float* p, size_t n, uint64_t seed, float mean, float stddev) {
  oracle_mt64 e;
  oracle_mt64_seed(&e, seed);
  const double two_pi = 6.283185307179586476925286766559;
  for (size_t i = 0; i < n; i += 2) {
    const double u1 = (double)(oracle_mt64_next(&e) >> 40) / (double)(1u << 24);
    const double u2 = (double)(oracle_mt64_next(&e) >> 40) / (double)(1u << 24);
    const double r = sqrt(-2.0 * log(1.0 - u1));
    p[i] = (float)((double)mean + (double)stddev * (r * cos(two_pi * u2)));
    if (i + 1 < n) p[i + 1] = (float)((double)mean + (double)stddev * (r * sin(two_pi * u2)));
  }
}

/* tests/reference.hpp:116-126. */
double oracle_gelu_erf(double x) { return 0.5 * x * (1.0 + erf(x * 0.70710678118654752440)); }

double oracle_gelu_tanh(double x) {
  const double k = 0.79788456080286535588;
  return 0.5 * x * (1.0 + tanh(k * (x + 0.044715 * x * x * x)));
}

/* tests/reference.hpp:128-136. */
static double apply_activation(double v, int act) {
  switch (act) {
    case ORACLE_ACT_NONE: return v;
    case ORACLE_ACT_RELU: return v > 0.0 ? v : 0.0;
    case ORACLE_ACT_GELU_ERF: return oracle_gelu_erf(v);
    case ORACLE_ACT_GELU_TANH: return oracle_gelu_tanh(v);
    default: return v;
  }
}

/* std::max(a, b) is (a < b) ? b : a: the first argument wins ties and any
 * comparison involving NaN, so a NaN element never replaces the running max. */
static double std_max(double a, double b) { return (a < b) ? b : a; }

/* tests/reference.hpp:143-151. */
void oracle_bias_act(const float* x, const float* bias, float* y, int64_t rows, int64_t cols,
                     int act) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      const double v = (double)x[r * cols + c] + (double)bias[c];
      y[r * cols + c] = (float)apply_activation(v, act);
    }
}

/* tests/reference.hpp:154-172. */
void oracle_row_reduce(const float* x, float* out, int64_t rows, int64_t cols, int kind) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* row = x + r * cols;
    if (kind == ORACLE_REDUCE_MAX) {
      double m = -INFINITY;
      for (int64_t c = 0; c < cols; ++c) m = std_max(m, (double)row[c]);
      out[r] = (float)m;
    } else {
      double s = 0.0;
      for (int64_t c = 0; c < cols; ++c) s += (double)row[c];
      if (kind == ORACLE_REDUCE_MEAN) s /= (double)cols;
      out[r] = (float)s;
    }
  }
}

/* tests/reference.hpp:175-191. */
void oracle_row_softmax(const float* x, float* y, int64_t rows, int64_t cols) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* row = x + r * cols;
    float* orow = y + r * cols;
    double m = -INFINITY;
    for (int64_t c = 0; c < cols; ++c) m = std_max(m, (double)row[c]);
    double sum = 0.0;
    for (int64_t c = 0; c < cols; ++c) sum += exp((double)row[c] - m);
    for (int64_t c = 0; c < cols; ++c) orow[c] = (float)(exp((double)row[c] - m) / sum);
  }
}

/* tests/reference.hpp:199-211.  Reads C even when beta == 0 (as the reference
 * does), so a NaN already in C propagates here; callers pass finite C. */
void oracle_gemm(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                 float alpha, float beta) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      double acc = 0.0;
      for (int64_t p = 0; p < k; ++p) acc += (double)a[i * k + p] * (double)b[p * n + j];
      const double prev = (double)c[i * n + j];
      c[i * n + j] = (float)((double)alpha * acc + (double)beta * prev);
    }
}

/* The full-vector case of tests/reference.hpp:154 (rows = 1): serial double sum
 * and a std::max fold; argmax added (unpinned by the reference). */
void oracle_full_reduce(const float* x, int64_t n, int64_t index_base, double* sum_out,
                        float* max_out, int64_t* argmax_out) {
  double s = 0.0;
  double m = -INFINITY;
  for (int64_t i = 0; i < n; ++i) {
    s += (double)x[i];
    m = std_max(m, (double)x[i]);
  }
  int64_t arg = -1;
  for (int64_t i = 0; i < n; ++i)
    if ((double)x[i] == m) { arg = i; break; }
  *sum_out = s;
  *max_out = (float)m;
  *argmax_out = arg < 0 ? -1 : arg + index_base;
}

/* Round-to-nearest-even float -> bfloat16 on the bit pattern. */
uint16_t oracle_f32_to_bf16(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0)
    return (uint16_t)((u >> 16) | 0x0040u);  /* quiet NaN */
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7FFFu + lsb;
  return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

void oracle_round_bf16(const float* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = oracle_bf16_to_f32(oracle_f32_to_bf16(in[i]));
}

void oracle_to_bf16(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = oracle_f32_to_bf16(in[i]);
}

/* tests/reference.hpp:344-347. */
double oracle_tol_gemm(int64_t k) {
  const double eps = 1.1920929e-7;
  return 4.0 * sqrt((double)(k < 1 ? 1 : k)) * eps;
}

/* tests/reference.hpp:370-374. */
double oracle_abs_tol_gemm(int64_t k, double amax) {
  const double eps = 1.1920929e-7;
  const double derived = 0.5 * (double)(k < 1 ? 1 : k) * eps * amax * amax / 3.0;
  return 3.0 * derived;
}

/* tests/reference.hpp:249-287 (mixed tolerance |g-w| <= abs + rel*|w|). */
size_t oracle_compare(const float* got, const float* want, size_t n, double rel_tol,
                      double abs_tol, double* max_abs_err, double* max_rel_err, int* any_nan,
                      int* any_inf) {
  size_t bad = 0;
  double mabs = 0.0, mrel = 0.0;
  int nan_seen = 0, inf_seen = 0;
  for (size_t i = 0; i < n; ++i) {
    const double g = (double)got[i];
    const double w = (double)want[i];
    if (isnan(g) || isnan(w)) { nan_seen = 1; ++bad; continue; }
    if ((isinf(g) != 0) != (isinf(w) != 0)) { inf_seen = 1; ++bad; continue; }
    const double ae = fabs(g - w);
    const double re = fabs(w) > 0.0 ? ae / fabs(w) : 0.0;
    if (ae > mabs) mabs = ae;
    if (re > mrel) mrel = re;
    if (ae > abs_tol + rel_tol * fabs(w)) ++bad;
  }
  if (max_abs_err) *max_abs_err = mabs;
  if (max_rel_err) *max_rel_err = mrel;
  if (any_nan) *any_nan = nan_seen;
  if (any_inf) *any_inf = inf_seen;
  return bad;
}

/* tests/reference.hpp:401-426. */
size_t oracle_spot_check_gemm(const float* a, const float* b, const float* got, int64_t m,
                              int64_t n, int64_t k, float alpha, size_t samples, uint64_t seed,
                              double rel_tol, double abs_tol, size_t* checked,
                              double* max_abs_err, double* max_rel_err) {
  size_t bad = 0, seen = 0;
  double mabs = 0.0, mrel = 0.0;
  if (m > 0 && n > 0 && k > 0) {
    oracle_mt64 rng;
    oracle_mt64_seed(&rng, seed);
    for (size_t s = 0; s < samples; ++s) {
      const int64_t i = (int64_t)(oracle_mt64_next(&rng) % (uint64_t)m);
      const int64_t j = (int64_t)(oracle_mt64_next(&rng) % (uint64_t)n);
      double acc = 0.0;
      for (int64_t p = 0; p < k; ++p) acc += (double)a[i * k + p] * (double)b[p * n + j];
      const double want = (double)alpha * acc;
      const double g = (double)got[i * n + j];
      ++seen;
      if (isnan(g) || isinf(g)) { ++bad; continue; }
      const double ae = fabs(g - want);
      const double re = fabs(want) > 0.0 ? ae / fabs(want) : 0.0;
      if (ae > mabs) mabs = ae;
      if (re > mrel) mrel = re;
      if (ae > abs_tol + rel_tol * fabs(want)) ++bad;
    }
  }
  if (checked) *checked = seen;
  if (max_abs_err) *max_abs_err = mabs;
  if (max_rel_err) *max_rel_err = mrel;
  return bad;
}
