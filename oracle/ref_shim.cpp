// C shim over the reference's torch-independent runtime core
// (ye3t/runtime/csrc/ye3t_runtime_core.{h,cpp}), which the Makefile compiles
// from the reference sources where they lie.  TEST INFRASTRUCTURE ONLY: used to
// pin the oracle restatement and as the reference CPU baseline in bench.py.
//
// Each wrapper splits its independent rows (edges or batch rows) into
// contiguous chunks over `threads` std::threads and calls the reference
// function once per chunk; the reference functions themselves are serial.

#include <complex>
#include <cstdint>
#include <thread>
#include <vector>

#include "ye3t_runtime_core.h"

namespace rt = ye3t::runtime;
using i64 = std::int64_t;

namespace {
template <typename F>
void chunks(i64 n, int threads, F body) {
  if (threads <= 1 || n < 2) { body(i64(0), n); return; }
  std::vector<std::thread> pool;
  const i64 step = (n + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    const i64 b = t * step, e = std::min<i64>(n, b + step);
    if (b >= e) break;
    pool.emplace_back([=] { body(b, e); });
  }
  for (auto& th : pool) th.join();
}
}  // namespace

extern "C" {

// ye3t_runtime_core.h:20 cheb_exp_cos_radial_table_with_derivative<double>
void yr_cheb_exp_cos_radial_table_f64(const double* r, const double* rc, const double* lam, i64 E,
                                      i64 kmax, double* val, double* der, int threads) {
  const i64 W = kmax + 1;
  chunks(E, threads, [&](i64 b, i64 e) {
    rt::cheb_exp_cos_radial_table_with_derivative<double>(r + b, rc + b, lam + b, e - b, kmax,
                                                          val + b * W, der + b * W);
  });
}

// ye3t_runtime_core.h:222 real_spherical_harmonics_table_with_derivative<double>
void yr_real_spherical_harmonics_table_f64(const double* vec, i64 E, i64 lmax, double eps,
                                           double* val, double* der, int threads) {
  const i64 W = (lmax + 1) * (lmax + 1);
  chunks(E, threads, [&](i64 b, i64 e) {
    rt::real_spherical_harmonics_table_with_derivative<double>(vec + 3 * b, e - b, lmax, eps,
                                                               val + b * W, der + 3 * b * W);
  });
}

// ye3t_runtime_core.h:109 complex_spherical_harmonics_table_with_derivative<double>
void yr_complex_spherical_harmonics_table_f64(const double* vec, i64 E, i64 lmax, double eps,
                                              double* val, double* der, int threads) {
  const i64 W = (lmax + 1) * (lmax + 1);
  auto* cv = reinterpret_cast<std::complex<double>*>(val);
  auto* cd = reinterpret_cast<std::complex<double>*>(der);
  chunks(E, threads, [&](i64 b, i64 e) {
    rt::complex_spherical_harmonics_table_with_derivative<double>(vec + 3 * b, e - b, lmax, eps,
                                                                  cv + b * W, cd + 3 * b * W);
  });
}

// ye3t_runtime_core.h:294 density_accumulate_forward (serial: one call)
void yr_density_accumulate_c128(const double* v, const i64* centers, i64 E, i64 C, i64 N,
                                double* out) {
  rt::density_accumulate_forward<std::complex<double>>(
      reinterpret_cast<const std::complex<double>*>(v), centers, E, C, N,
      reinterpret_cast<std::complex<double>*>(out));
}

void yr_density_accumulate_f64(const double* v, const i64* centers, i64 E, i64 C, i64 N,
                               double* out) {
  rt::density_accumulate_forward<double>(v, centers, E, C, N, out);
}

// ye3t_runtime_core.h:1227 symmetric_power_monomial_forward
void yr_symmetric_power_monomial_c128(const double* x, i64 batch, i64 in_dim, const i64* counts,
                                      const i64* off, const double* values, i64 terms,
                                      i64 out_dim, double* out, int threads) {
  const auto* cx = reinterpret_cast<const std::complex<double>*>(x);
  const auto* cvals = reinterpret_cast<const std::complex<double>*>(values);
  auto* co = reinterpret_cast<std::complex<double>*>(out);
  chunks(batch, threads, [&](i64 b, i64 e) {
    rt::symmetric_power_monomial_forward<std::complex<double>>(
        cx + b * in_dim, e - b, in_dim, counts, off, cvals, terms, out_dim, co + b * out_dim);
  });
}

void yr_symmetric_power_monomial_f64(const double* x, i64 batch, i64 in_dim, const i64* counts,
                                     const i64* off, const double* values, i64 terms, i64 out_dim,
                                     double* out, int threads) {
  chunks(batch, threads, [&](i64 b, i64 e) {
    rt::symmetric_power_monomial_forward<double>(x + b * in_dim, e - b, in_dim, counts, off,
                                                 values, terms, out_dim, out + b * out_dim);
  });
}


// ye3t_runtime_core.h:76 pace_radial_channel_contraction_with_derivative (serial: one call)
void yr_pace_radial_channel_contraction_f64(const double* in, const double* din, const double* W, i64 P, i64 I,
                                            i64 O, double* out, double* dout) {
  rt::pace_radial_channel_contraction_with_derivative<double>(in, din, W, P, I, O, out, dout);
}

void yr_pace_radial_channel_contraction_f32(const float* in, const float* din, const float* W, i64 P, i64 I,
                                            i64 O, float* out, float* dout) {
  rt::pace_radial_channel_contraction_with_derivative<float>(in, din, W, P, I, O, out, dout);
}
}  // extern "C"
