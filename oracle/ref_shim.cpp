// oracle/ref_shim.cpp -- C linkage for the reference's own CPU oracle.
//
// TEST INFRASTRUCTURE ONLY.  This file contains no arithmetic: it includes the
// reference's header-only CPU oracle, mini-cuda-kernel-engine
// tests/reference.hpp, from the reference's source tree (it is never copied
// here) and gives each function an extern "C" name so that Python can call it
// through ctypes.  oracle/Makefile builds it into oracle/_ref/libmcke_ref.so,
// which is git-ignored and travels to the GPU box with the rest of the tree.
//
// Uses:
//   * tests/test_oracle.py pins the C restatement in oracle/mcke_oracle.c
//     against it, function by function, bit for bit;
//   * tests/golden/make_golden.py generates the committed fixtures from it;
//   * bench.py's reference arm and cpu_baseline leg time it on the host cores.
#include <cstddef>
#include <cstdint>

#include "reference.hpp"

namespace t = mcke::testing;
namespace k = mcke::kernels;

extern "C" {

// tests/reference.hpp:101
void ref_fill_random(float* p, std::size_t n, std::uint64_t seed, float lo, float hi) {
  t::fill_random(p, n, seed, lo, hi);
}

// tests/reference.hpp:116, :121
double ref_gelu_erf(double x) { return t::gelu_erf(x); }
double ref_gelu_tanh(double x) { return t::gelu_tanh(x); }

// tests/reference.hpp:143
void ref_bias_act(const float* x, const float* bias, float* y, std::int64_t rows,
                  std::int64_t cols, int act) {
  t::reference_bias_act(x, bias, y, rows, cols, static_cast<k::Activation>(act));
}

// tests/reference.hpp:154
void ref_row_reduce(const float* x, float* out, std::int64_t rows, std::int64_t cols, int kind) {
  t::reference_row_reduce(x, out, rows, cols, static_cast<k::ReduceKind>(kind));
}

// tests/reference.hpp:175
void ref_row_softmax(const float* x, float* y, std::int64_t rows, std::int64_t cols) {
  t::reference_row_softmax(x, y, rows, cols);
}

// tests/reference.hpp:199
void ref_gemm(const float* a, const float* b, float* c, std::int64_t m, std::int64_t n,
              std::int64_t kk, float alpha, float beta) {
  t::reference_gemm(a, b, c, m, n, kk, alpha, beta);
}

// tests/reference.hpp:249
std::size_t ref_compare(const float* got, const float* want, std::size_t n, double rel_tol,
                        double abs_tol, double* max_abs_err, double* max_rel_err, int* any_nan,
                        int* any_inf) {
  const t::CompareResult r = t::compare(got, want, n, rel_tol, abs_tol);
  if (max_abs_err) *max_abs_err = r.max_abs_err;
  if (max_rel_err) *max_rel_err = r.max_rel_err;
  if (any_nan) *any_nan = r.any_nan ? 1 : 0;
  if (any_inf) *any_inf = r.any_inf ? 1 : 0;
  return r.mismatches;
}

// tests/reference.hpp:344, :370
double ref_tol_gemm(std::int64_t kk) { return t::tol_gemm(kk); }
double ref_abs_tol_gemm(std::int64_t kk, double amax) { return t::abs_tol_gemm(kk, amax); }

// tests/reference.hpp:401
std::size_t ref_spot_check_gemm(const float* a, const float* b, const float* got,
                                std::int64_t m, std::int64_t n, std::int64_t kk, float alpha,
                                std::size_t samples, std::uint64_t seed, double rel_tol,
                                double abs_tol, std::size_t* checked, double* max_abs_err,
                                double* max_rel_err) {
  const t::SpotCheckResult r =
      t::spot_check_gemm(a, b, got, m, n, kk, alpha, samples, seed, rel_tol, abs_tol);
  if (checked) *checked = r.checked;
  if (max_abs_err) *max_abs_err = r.max_abs_err;
  if (max_rel_err) *max_rel_err = r.max_rel_err;
  return r.mismatches;
}

}  // extern "C"
