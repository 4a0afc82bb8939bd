/*
 * oracle/mcke_oracle.h -- CPU restatement of the reference's CPU oracle.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code.  It exists so that tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py can check the CUDA kernels against an
 * independent CPU answer.  The product path fails loudly when its CUDA
 * extension is missing; it never routes through this file.
 *
 * Every function restates one function of the reference's header-only CPU
 * oracle, mini-cuda-kernel-engine tests/reference.hpp, and cites the line it
 * follows.  Arithmetic is kept in the same order and the same precision
 * (double accumulation, float storage) so that the restatement agrees with the
 * compiled reference bit for bit; tests/test_oracle.py checks exactly that,
 * against the reference's own golden vectors (tests/data/reference_vectors.txt,
 * converted into tests/golden/reference_vectors.json) and against the
 * reference itself compiled into oracle/_ref/.
 *
 * Three functions have no counterpart in the reference and are therefore
 * "parity unpinned" by its tests:
 *   - oracle_full_reduce's argmax (lowest index on ties),
 *   - oracle_fill_normal (Box-Muller over fill_random's 24-bit uniforms),
 *   - oracle_round_bf16 (round-to-nearest-even to bfloat16).
 * Their sum/max halves and their building blocks are pinned.
 */
#ifndef MCKE_ORACLE_H_
#define MCKE_ORACLE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Activation / reduce-kind numbering follows the reference's enums
 * (include/mcke/kernels/kernels.hpp:65 and :153). */
enum { ORACLE_ACT_NONE = 0, ORACLE_ACT_RELU = 1, ORACLE_ACT_GELU_ERF = 2, ORACLE_ACT_GELU_TANH = 3 };
enum { ORACLE_REDUCE_SUM = 0, ORACLE_REDUCE_MAX = 1, ORACLE_REDUCE_MEAN = 2 };

/* mt19937_64 engine (Matsumoto & Nishimura, 64-bit variant; the parameters the
 * C++ standard fixes for std::mt19937_64). */
typedef struct {
  uint64_t mt[312];
  int idx;
} oracle_mt64;

void oracle_mt64_seed(oracle_mt64* e, uint64_t seed);
uint64_t oracle_mt64_next(oracle_mt64* e);

/* tests/reference.hpp:101 fill_random. */
void oracle_fill_random(float* p, size_t n, uint64_t seed, float lo, float hi);
/* Builder convention (unpinned): N(mean, stddev^2) by Box-Muller. */
void oracle_fill_normal(float* p, size_t n, uint64_t seed, float mean, float stddev);

/* tests/reference.hpp:116 and :121. */
double oracle_gelu_erf(double x);
double oracle_gelu_tanh(double x);

/* tests/reference.hpp:143 reference_bias_act. */
void oracle_bias_act(const float* x, const float* bias, float* y, int64_t rows, int64_t cols,
                     int act);
/* tests/reference.hpp:154 reference_row_reduce. */
void oracle_row_reduce(const float* x, float* out, int64_t rows, int64_t cols, int kind);
/* tests/reference.hpp:175 reference_row_softmax. */
void oracle_row_softmax(const float* x, float* y, int64_t rows, int64_t cols);
/* tests/reference.hpp:199 reference_gemm. */
void oracle_gemm(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                 float alpha, float beta);

/* Full-vector reduce: sum (double, serial, as reference_row_reduce with rows=1),
 * max (std::max fold from -inf, so NaN elements are skipped) and argmax = the
 * lowest index i with x[i] == max (-1 when no element compares >= -inf, i.e.
 * n == 0 or every element is NaN).  `index_base` is added to the returned
 * index so a shard can report global positions. */
void oracle_full_reduce(const float* x, int64_t n, int64_t index_base, double* sum_out,
                        float* max_out, int64_t* argmax_out);

/* float -> bfloat16 with round-to-nearest-even (NaN kept quiet).  The _round
 * form writes the bf16 value widened back to float. */
uint16_t oracle_f32_to_bf16(float v);
float oracle_bf16_to_f32(uint16_t h);
void oracle_round_bf16(const float* in, float* out, size_t n);
void oracle_to_bf16(const float* in, uint16_t* out, size_t n);

/* tests/reference.hpp:344 tol_gemm and :370 abs_tol_gemm. */
double oracle_tol_gemm(int64_t k);
double oracle_abs_tol_gemm(int64_t k, double amax);

/* tests/reference.hpp:249 compare.  Returns the mismatch count; fills the
 * maxima and NaN/Inf flags. */
size_t oracle_compare(const float* got, const float* want, size_t n, double rel_tol,
                      double abs_tol, double* max_abs_err, double* max_rel_err, int* any_nan,
                      int* any_inf);

/* tests/reference.hpp:401 spot_check_gemm (beta assumed 0).  Returns the
 * mismatch count; `checked` and the maxima are filled. */
size_t oracle_spot_check_gemm(const float* a, const float* b, const float* got, int64_t m,
                              int64_t n, int64_t k, float alpha, size_t samples, uint64_t seed,
                              double rel_tol, double abs_tol, size_t* checked,
                              double* max_abs_err, double* max_rel_err);

#ifdef __cplusplus
}
#endif
#endif /* MCKE_ORACLE_H_ */
