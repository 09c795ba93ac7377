// CPU oracle for the ye3t ACE feature path.
//
// TEST INFRASTRUCTURE ONLY.  This file restates, in plain serial C++, the
// reference algorithms that the CUDA library in ye3t_b200/csrc replaces.  It
// is loaded only by tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline leg, always as the checker or the timed CPU baseline and never as
// a product code path.  Each function cites the reference file:line whose
// behaviour it follows (paths relative to the ye3t project root).
//
// Complex values use std::complex<T>, which is layout-compatible with numpy's
// complex64 / complex128 (interleaved re, im).
//
// dtype codes used by every entry point: 0 = float32, 1 = float64,
// 2 = complex64, 3 = complex128.

#include <algorithm>
#include <cmath>
#include <complex>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

using i64 = std::int64_t;
using c64 = std::complex<float>;
using c128 = std::complex<double>;

namespace {

// Persistent worker pool behind parallel_chunks.  The reference's CPU
// evaluator runs on at::parallel_for, whose threads live for the whole
// process; starting threads per call instead would cost more than the work of
// a small batch.  Workers sleep on a condition variable between calls; one
// parallel call runs at a time (callers are serialised); the pool is never
// destroyed, so process exit does not wait on it.
class ChunkPool {
 public:
  static ChunkPool& get() {
    static ChunkPool* pool = new ChunkPool();
    return *pool;
  }

  // Runs job(0) .. job(T - 1), job(0) on the calling thread.
  void run(int T, const std::function<void(int)>& job) {
    std::lock_guard<std::mutex> call(call_mu_);
    std::unique_lock<std::mutex> lk(mu_);
    while (static_cast<int>(workers_.size()) < T - 1) {
      const int index = static_cast<int>(workers_.size()) + 1;
      const std::uint64_t seen = gen_;
      workers_.emplace_back([this, index, seen] { loop(index, seen); });
    }
    job_ = &job;
    participants_ = T - 1;
    remaining_ = T - 1;
    ++gen_;
    lk.unlock();
    wake_.notify_all();
    job(0);
    lk.lock();
    done_.wait(lk, [&] { return remaining_ == 0; });
    job_ = nullptr;
  }

 private:
  void loop(int index, std::uint64_t seen) {
    std::unique_lock<std::mutex> lk(mu_);
    for (;;) {
      wake_.wait(lk, [&] { return gen_ != seen; });
      seen = gen_;
      if (index > participants_) continue;
      const std::function<void(int)>* job = job_;
      lk.unlock();
      (*job)(index);
      lk.lock();
      if (--remaining_ == 0) done_.notify_one();
    }
  }

  std::mutex call_mu_, mu_;
  std::condition_variable wake_, done_;
  std::vector<std::thread> workers_;
  const std::function<void(int)>* job_ = nullptr;
  std::uint64_t gen_ = 0;
  int participants_ = 0, remaining_ = 0;
};

// Runs body(begin, end) over [0, n) split into `threads` contiguous chunks
// (one chunk per thread, as at::parallel_for with grain 0).
template <typename F>
void parallel_chunks(std::int64_t n, int threads, F body) {
  if (threads <= 1 || n < 2) { body(std::int64_t(0), n); return; }
  const int T = static_cast<int>(std::min<std::int64_t>(threads, n));
  const std::int64_t step = (n + T - 1) / T;
  const std::function<void(int)> job = [&](int t) {
    const std::int64_t b = t * step, e = std::min<std::int64_t>(n, b + step);
    if (b < e) body(b, e);
  };
  ChunkPool::get().run(T, job);
}

// ---------------------------------------------------------------------------
// Factorized schedule evaluation.
// Follows ye3t/core/csrc/factorized_runtime.cpp:252-287 (evaluate_componentwise)
// and the torch path ye3t/core/couplings.py:552-567:
//   out[b, c] = sum_{t in [off[c], off[c+1])} coeff[t] *
//               prod_j bv[b, label[c], j, m_idx[t, j]]
// The product starts from the coefficient and multiplies blocks in order; the
// accumulation runs over terms in table order, as in the reference C++ loop.
// ---------------------------------------------------------------------------
template <typename S>
void schedule_eval(const S* bv, i64 batch, i64 basis, i64 blocks, i64 mdim,
                   const i64* off, const i64* labels, const i64* midx,
                   const S* coeffs, i64 comps, S* out, int threads) {
  parallel_chunks(batch * comps, threads, [&](i64 lo, i64 hi) {
  for (i64 lin = lo; lin < hi; ++lin) {
    const i64 b = lin / comps;
    const i64 c = lin - b * comps;
    const i64 label = labels[c];
    const S* row = bv + (b * basis + label) * blocks * mdim;
    S acc = S(0);
    for (i64 t = off[c]; t < off[c + 1]; ++t) {
      S v = coeffs[t];
      for (i64 j = 0; j < blocks; ++j) v *= row[j * mdim + midx[t * blocks + j]];
      acc += v;
    }
    out[lin] = acc;
  }
  });
}

// ---------------------------------------------------------------------------
// Symmetric-power monomial contraction (grouped table).
// Follows ye3t/runtime/csrc/ye3t_runtime_core.cpp:5279 and the torch
// reference ye3t/runtime/execution_plan.py:11894:
//   out[b, o] = sum_{t in [off[o], off[o+1])} value[t] * prod_i x[b,i]^count[t,i]
// Integer powers are formed by repeated multiplication.
// ---------------------------------------------------------------------------
template <typename S>
S ipow(S x, i64 e) {
  S r = S(1);
  for (i64 k = 0; k < e; ++k) r *= x;
  return r;
}

template <typename S>
void sympow(const S* x, i64 batch, i64 in_dim, const i64* counts, const i64* off,
            const S* values, i64 out_dim, S* out) {
  for (i64 b = 0; b < batch; ++b) {
    const S* xr = x + b * in_dim;
    for (i64 o = 0; o < out_dim; ++o) {
      S acc = S(0);
      for (i64 t = off[o]; t < off[o + 1]; ++t) {
        S m = values[t];
        for (i64 i = 0; i < in_dim; ++i) m *= ipow(xr[i], counts[t * in_dim + i]);
        acc += m;
      }
      out[b * out_dim + o] = acc;
    }
  }
}

// Shared-monomial form: unique monomials first, then a sparse coefficient map.
// Follows ye3t/runtime/csrc/ye3t_runtime_core.cpp:5392 (output row o collects
// coefficient entries [off[o], off[o+1]) each naming one unique monomial).
template <typename S>
void sympow_shared(const S* x, i64 batch, i64 in_dim, const i64* counts, i64 mono,
                   const i64* off, const i64* terms, const S* values, i64 out_dim,
                   S* out) {
  std::vector<S> m(mono);
  for (i64 b = 0; b < batch; ++b) {
    const S* xr = x + b * in_dim;
    for (i64 u = 0; u < mono; ++u) {
      S p = S(1);
      for (i64 i = 0; i < in_dim; ++i) p *= ipow(xr[i], counts[u * in_dim + i]);
      m[u] = p;
    }
    for (i64 o = 0; o < out_dim; ++o) {
      S acc = S(0);
      for (i64 c = off[o]; c < off[o + 1]; ++c) acc += values[c] * m[terms[c]];
      out[b * out_dim + o] = acc;
    }
  }
}

// ---------------------------------------------------------------------------
// ChebExpCos radial basis with d/dr.
// Follows ye3t/runtime/csrc/ye3t_runtime_core.cpp:320-392 and the torch
// reference ye3t/runtime/execution_plan.py:6862-6891:
//   s = r / max(rc, eps);  zero for s > 1
//   k = 0: 1;  k = 1: (1 + cos(pi s)) / 2
//   k >= 2: (1 - T_k(x)) (1 + cos(pi s)) / 4,
//           x = 1 - 2 expm1(-lambda (s - 1)) / expm1(lambda)
// ---------------------------------------------------------------------------
template <typename R>
void radial_one(R r, R rc_in, R lam, i64 kmax, R* val, R* der) {
  const R pi = std::acos(R(-1));
  const R rc = std::max(rc_in, std::numeric_limits<R>::epsilon());
  const R s = r / rc;
  for (i64 k = 0; k <= kmax; ++k) { val[k] = R(0); der[k] = R(0); }
  if (s > R(1)) return;
  val[0] = R(1);
  const R env = R(1) + std::cos(pi * s);
  const R denv = -pi * std::sin(pi * s) / rc;
  if (kmax >= 1) {
    val[1] = R(0.5) * env;
    der[1] = R(0.5) * denv;
  }
  if (kmax < 2) return;
  const R ex = std::exp(-lam * (s - R(1)));
  const R den = std::expm1(lam);
  const R x = R(1) - R(2) * std::expm1(-lam * (s - R(1))) / den;
  const R dx = R(2) * lam * ex / (den * rc);
  // Chebyshev T_k(x) and T'_k(x) = k U_{k-1}(x) by forward recurrence.
  R t0 = R(1), t1 = x;      // T_0, T_1
  R u0 = R(1), u1 = R(2) * x;  // U_0, U_1
  for (i64 k = 2; k <= kmax; ++k) {
    const R t2 = R(2) * x * t1 - t0;
    t0 = t1; t1 = t2;          // t1 = T_k
    // u1 holds U_{k-1} here, so T'_k = k U_{k-1}.
    const R dT = R(k) * u1;
    val[k] = R(0.25) * (R(1) - t1) * env;
    der[k] = R(0.25) * (-dT * dx * env + (R(1) - t1) * denv);
    const R u2 = R(2) * x * u1 - u0;
    u0 = u1; u1 = u2;
  }
}

// ---------------------------------------------------------------------------
// Real spherical harmonics on the unit sphere, with the gradient of their
// polynomial extension in (ux, uy, uz).
// Follows the convention of ye3t/runtime/csrc/ye3t_runtime_core.cpp:226-290
// and ye3t/core/spherical.py:113-170:
//   Y_{l,0}  = N_{l0} Q_l^0(uz)
//   Y_{l,+m} =  sqrt2 N_{lm} Q_l^m(uz) Re((ux + i uy)^m)
//   Y_{l,-m} = -sqrt2 N_{lm} Q_l^m(uz) Im((ux + i uy)^m)
// with Q_l^m = d^m P_l / dz^m and N_{lm} = sqrt((2l+1)/(4 pi) (l-m)!/(l+m)!).
// Q_l^m is evaluated here by the fixed-m three-term recurrence in l
//   Q_m^m = (2m-1)!!,  Q_{m+1}^m = (2m+1) z Q_m^m,
//   (l-m) Q_l^m = (2l-1) z Q_{l-1}^m - (l+m-1) Q_{l-2}^m,
// and dQ_l^m/dz = Q_l^{m+1}.
// ---------------------------------------------------------------------------
template <typename R>
R qlm(i64 l, i64 m, R z) {
  if (m > l) return R(0);
  R qmm = R(1);
  for (i64 k = 1; k <= m; ++k) qmm *= R(2 * k - 1);
  if (l == m) return qmm;
  R qa = qmm, qb = R(2 * m + 1) * z * qmm;
  for (i64 ll = m + 2; ll <= l; ++ll) {
    const R qc = (R(2 * ll - 1) * z * qb - R(ll + m - 1) * qa) / R(ll - m);
    qa = qb; qb = qc;
  }
  return qb;
}

template <typename R>
R norm_lm(i64 l, i64 m) {
  const double v = 0.5 * (std::log(2.0 * l + 1.0) - std::log(4.0 * M_PI) +
                          std::lgamma(double(l - m + 1)) - std::lgamma(double(l + m + 1)));
  return R(std::exp(v));
}

template <typename R>
void real_sh_unit(i64 l, R ux, R uy, R uz, R* val, R* grad) {
  const i64 w = 2 * l + 1;
  for (i64 i = 0; i < w; ++i) { val[i] = R(0); grad[3 * i] = grad[3 * i + 1] = grad[3 * i + 2] = R(0); }
  const R n0 = norm_lm<R>(l, 0);
  val[l] = n0 * qlm<R>(l, 0, uz);
  grad[3 * l + 2] = n0 * qlm<R>(l, 1, uz);
  const R rt2 = std::sqrt(R(2));
  std::complex<R> pw(R(1), R(0)), prev(R(1), R(0));
  const std::complex<R> xy(ux, uy);
  for (i64 m = 1; m <= l; ++m) {
    prev = pw;
    pw *= xy;
    const R q = qlm<R>(l, m, uz);
    const R dq = qlm<R>(l, m + 1, uz);
    const R sc = rt2 * norm_lm<R>(l, m);
    const i64 p = l + m, n = l - m;
    // d/dux (ux+i uy)^m = m (ux+i uy)^(m-1);  d/duy = i m (ux+i uy)^(m-1)
    val[p] = sc * q * pw.real();
    grad[3 * p + 0] = sc * q * (R(m) * prev.real());
    grad[3 * p + 1] = sc * q * (-R(m) * prev.imag());
    grad[3 * p + 2] = sc * dq * pw.real();
    val[n] = -sc * q * pw.imag();
    grad[3 * n + 0] = -sc * q * (R(m) * prev.imag());
    grad[3 * n + 1] = -sc * q * (R(m) * prev.real());
    grad[3 * n + 2] = -sc * dq * pw.imag();
  }
}

// Edge-vector table with Cartesian derivatives.  The unit-vector Jacobian
// (I - u u^T)/|r| (or I/eps below eps) follows
// ye3t/runtime/csrc/ye3t_runtime_core.cpp:797-840.  The complex table is
// built from the real one exactly as ye3t_runtime_core.cpp:891-948:
//   Yc_{l,-m} = (R_{+m} + i R_{-m}) / sqrt2,
//   Yc_{l,+m} = (-1)^m (R_{+m} - i R_{-m}) / sqrt2.
template <typename R>
void sh_table(const R* vec, i64 E, i64 lmax, bool real_out, R eps, void* val_out, void* der_out) {
  const i64 W = (lmax + 1) * (lmax + 1);
  std::vector<R> v(2 * lmax + 1), g(3 * (2 * lmax + 1));
  R* rv = static_cast<R*>(val_out);
  R* rd = static_cast<R*>(der_out);
  auto* cv = static_cast<std::complex<R>*>(val_out);
  auto* cd = static_cast<std::complex<R>*>(der_out);
  const R inv2 = R(1) / std::sqrt(R(2));
  for (i64 e = 0; e < E; ++e) {
    const R x = vec[3 * e], y = vec[3 * e + 1], z = vec[3 * e + 2];
    const R r = std::sqrt(x * x + y * y + z * z);
    const R sr = std::max(r, eps);
    const R u[3] = {x / sr, y / sr, z / sr};
    R jac[3][3];
    for (int a = 0; a < 3; ++a)
      for (int b = 0; b < 3; ++b) {
        if (r > eps) jac[a][b] = ((a == b ? R(1) : R(0)) - u[a] * u[b]) / sr;
        else jac[a][b] = (a == b) ? R(1) / sr : R(0);
      }
    for (i64 l = 0; l <= lmax; ++l) {
      real_sh_unit<R>(l, u[0], u[1], u[2], v.data(), g.data());
      const i64 w = 2 * l + 1;
      std::vector<R> dvv(3 * w);
      for (i64 i = 0; i < w; ++i)
        for (int a = 0; a < 3; ++a) {
          R s = R(0);
          for (int b = 0; b < 3; ++b) s += g[3 * i + b] * jac[a][b];
          dvv[3 * i + a] = s;
        }
      const i64 base = e * W + l * l;
      if (real_out) {
        for (i64 i = 0; i < w; ++i) {
          rv[base + i] = v[i];
          for (int a = 0; a < 3; ++a) rd[3 * (base + i) + a] = dvv[3 * i + a];
        }
      } else {
        cv[base + l] = std::complex<R>(v[l], R(0));
        for (int a = 0; a < 3; ++a) cd[3 * (base + l) + a] = std::complex<R>(dvv[3 * l + a], R(0));
        for (i64 m = 1; m <= l; ++m) {
          const i64 p = l + m, n = l - m;
          const R sg = (m % 2 == 0) ? R(1) : R(-1);
          cv[base + n] = inv2 * std::complex<R>(v[p], v[n]);
          cv[base + p] = sg * inv2 * std::complex<R>(v[p], -v[n]);
          for (int a = 0; a < 3; ++a) {
            cd[3 * (base + n) + a] = inv2 * std::complex<R>(dvv[3 * p + a], dvv[3 * n + a]);
            cd[3 * (base + p) + a] = sg * inv2 * std::complex<R>(dvv[3 * p + a], -dvv[3 * n + a]);
          }
        }
      }
    }
  }
}

// Density accumulation, ye3t/runtime/csrc/ye3t_runtime_core.cpp:1684:
//   A[centers[e], c] += v[e, c], edges in index order.
template <typename S>
void density(const S* v, const i64* centers, i64 E, i64 C, i64 N, S* out) {
  std::fill(out, out + N * C, S(0));
  for (i64 e = 0; e < E; ++e) {
    const i64 i = centers[e];
    for (i64 c = 0; c < C; ++c) out[i * C + c] += v[e * C + c];
  }
}

template <typename S>
void density_adjoint(const S* adj, const i64* centers, i64 E, i64 C, S* out) {
  for (i64 e = 0; e < E; ++e)
    for (i64 c = 0; c < C; ++c) out[e * C + c] = adj[centers[e] * C + c];
}

template <typename R>
void contraction(const R* in, const R* din, const R* W, i64 P, i64 I, i64 O, R* out, R* dout) {
  for (i64 p = 0; p < P; ++p)
    for (i64 o = 0; o < O; ++o) {
      R v = R(0), d = R(0);
      for (i64 i = 0; i < I; ++i) {
        const R c = W[o * I + i];
        const R a = c * in[p * I + i];
        const R b = c * din[p * I + i];
        v = v + a;
        d = d + b;
      }
      out[p * O + o] = v;
      dout[p * O + o] = d;
    }
}

}  // namespace

extern "C" {

int yo_version(void) { return 1; }

void yo_factorized_schedule_evaluate(int dtype, const void* bv, i64 batch, i64 basis, i64 blocks,
                                     i64 mdim, const i64* off, const i64* labels, const i64* midx,
                                     const void* coeffs, i64 comps, void* out, int threads) {
  if (threads < 1) threads = 1;
  switch (dtype) {
    case 0: schedule_eval((const float*)bv, batch, basis, blocks, mdim, off, labels, midx, (const float*)coeffs, comps, (float*)out, threads); break;
    case 1: schedule_eval((const double*)bv, batch, basis, blocks, mdim, off, labels, midx, (const double*)coeffs, comps, (double*)out, threads); break;
    case 2: schedule_eval((const c64*)bv, batch, basis, blocks, mdim, off, labels, midx, (const c64*)coeffs, comps, (c64*)out, threads); break;
    case 3: schedule_eval((const c128*)bv, batch, basis, blocks, mdim, off, labels, midx, (const c128*)coeffs, comps, (c128*)out, threads); break;
  }
}

void yo_symmetric_power_monomial(int dtype, const void* x, i64 batch, i64 in_dim, const i64* counts,
                                 const i64* off, const void* values, i64 out_dim, void* out) {
  switch (dtype) {
    case 0: sympow((const float*)x, batch, in_dim, counts, off, (const float*)values, out_dim, (float*)out); break;
    case 1: sympow((const double*)x, batch, in_dim, counts, off, (const double*)values, out_dim, (double*)out); break;
    case 2: sympow((const c64*)x, batch, in_dim, counts, off, (const c64*)values, out_dim, (c64*)out); break;
    case 3: sympow((const c128*)x, batch, in_dim, counts, off, (const c128*)values, out_dim, (c128*)out); break;
  }
}

void yo_symmetric_power_shared_monomial(int dtype, const void* x, i64 batch, i64 in_dim,
                                        const i64* counts, i64 mono, const i64* off,
                                        const i64* terms, const void* values, i64 out_dim,
                                        void* out) {
  switch (dtype) {
    case 0: sympow_shared((const float*)x, batch, in_dim, counts, mono, off, terms, (const float*)values, out_dim, (float*)out); break;
    case 1: sympow_shared((const double*)x, batch, in_dim, counts, mono, off, terms, (const double*)values, out_dim, (double*)out); break;
    case 2: sympow_shared((const c64*)x, batch, in_dim, counts, mono, off, terms, (const c64*)values, out_dim, (c64*)out); break;
    case 3: sympow_shared((const c128*)x, batch, in_dim, counts, mono, off, terms, (const c128*)values, out_dim, (c128*)out); break;
  }
}

void yo_cheb_exp_cos_radial_table(int dtype, const void* r, const void* rc, const void* lam, i64 E,
                                  i64 kmax, void* val, void* der) {
  const i64 W = kmax + 1;
  if (dtype == 1) {
    for (i64 e = 0; e < E; ++e)
      radial_one<double>(((const double*)r)[e], ((const double*)rc)[e], ((const double*)lam)[e], kmax,
                         (double*)val + e * W, (double*)der + e * W);
  } else {
    for (i64 e = 0; e < E; ++e)
      radial_one<float>(((const float*)r)[e], ((const float*)rc)[e], ((const float*)lam)[e], kmax,
                        (float*)val + e * W, (float*)der + e * W);
  }
}

void yo_spherical_harmonics_table(int dtype, const void* vec, i64 E, i64 lmax, int real_output,
                                  double eps, void* val, void* der) {
  if (dtype == 1) sh_table<double>((const double*)vec, E, lmax, real_output != 0, eps, val, der);
  else sh_table<float>((const float*)vec, E, lmax, real_output != 0, (float)eps, val, der);
}

void yo_density_accumulate(int dtype, const void* v, const i64* centers, i64 E, i64 C, i64 N, void* out) {
  switch (dtype) {
    case 0: density((const float*)v, centers, E, C, N, (float*)out); break;
    case 1: density((const double*)v, centers, E, C, N, (double*)out); break;
    case 2: density((const c64*)v, centers, E, C, N, (c64*)out); break;
    case 3: density((const c128*)v, centers, E, C, N, (c128*)out); break;
  }
}

void yo_density_accumulate_adjoint(int dtype, const void* adj, const i64* centers, i64 E, i64 C, void* out) {
  switch (dtype) {
    case 0: density_adjoint((const float*)adj, centers, E, C, (float*)out); break;
    case 1: density_adjoint((const double*)adj, centers, E, C, (double*)out); break;
    case 2: density_adjoint((const c64*)adj, centers, E, C, (c64*)out); break;
    case 3: density_adjoint((const c128*)adj, centers, E, C, (c128*)out); break;
  }
}

// Brute-force periodic minimum-image neighbour list in CSR form.  The
// reference has no neighbour-list code; this is the test oracle for the CUDA
// cell-list builder.  Row i lists every j != i with |r_j - r_i|_mic <= rc in
// increasing j.  Returns the edge count, or -1 when cap is too small.
i64 yo_neighbor_list_bruteforce(const double* pos, i64 N, double box, double rc, i64* row_off,
                                int* nbr, double* disp, i64 cap) {
  i64 e = 0;
  const double rc2 = rc * rc;
  row_off[0] = 0;
  for (i64 i = 0; i < N; ++i) {
    for (i64 j = 0; j < N; ++j) {
      if (j == i) continue;
      double d[3];
      for (int a = 0; a < 3; ++a) {
        double x = pos[3 * j + a] - pos[3 * i + a];
        x -= box * std::nearbyint(x / box);
        d[a] = x;
      }
      const double r2 = d[0] * d[0] + d[1] * d[1] + d[2] * d[2];
      if (r2 <= rc2) {
        if (e >= cap) return -1;
        nbr[e] = (int)j;
        if (disp) { disp[3 * e] = d[0]; disp[3 * e + 1] = d[1]; disp[3 * e + 2] = d[2]; }
        ++e;
      }
    }
    row_off[i + 1] = e;
  }
  return e;
}

// ACE atomic density (A-basis) over a CSR neighbour list, the composition of
// ye3t/runtime/execution_plan.py:7298 (radial table), :7479 (complex
// harmonics, real_output=False), a per-neighbour-species prefactor as in
// plain_site_basis_product (:7582) and density_accumulate (:7913):
//   A[i, n-1, l^2 + l + m] = sum_{e in row i} p[z_{nbr[e]}] R_n(|d_e|) Yc_lm(d_e)
// for radial indices n = 1..nmax.  Edges are summed in CSR order.
void yo_ace_density(const double* disp, const i64* row_off, const int* nbr, const int* species,
                    const double* prefactor, i64 N, i64 nmax, i64 lmax, double rc, double lam,
                    double* A_out /* complex128 [N, nmax, (lmax+1)^2] */) {
  const i64 W = (lmax + 1) * (lmax + 1);
  c128* A = reinterpret_cast<c128*>(A_out);
  std::vector<double> rv(nmax + 1), rd(nmax + 1);
  std::vector<c128> yv(W), yd(3 * W);
  for (i64 i = 0; i < N; ++i) {
    c128* Ai = A + i * nmax * W;
    for (i64 k = 0; k < nmax * W; ++k) Ai[k] = c128(0, 0);
    for (i64 e = row_off[i]; e < row_off[i + 1]; ++e) {
      const double* d = disp + 3 * e;
      const double r = std::sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
      radial_one<double>(r, rc, lam, nmax, rv.data(), rd.data());
      sh_table<double>(d, 1, lmax, false, 1e-12, yv.data(), yd.data());
      const double p = prefactor[species[nbr[e]]];
      for (i64 n = 1; n <= nmax; ++n) {
        const double pr = p * rv[n];
        for (i64 k = 0; k < W; ++k) Ai[(n - 1) * W + k] += pr * yv[k];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Force path (complex128 only).  The reference obtains these by torch
// autograd: through the gather-and-product schedule evaluator
// (ye3t/core/couplings.py:552-567), the symmetric-power contraction
// (ye3t/runtime/execution_plan.py:11998) and the edge products
// (plain_site_basis_product, :7582; density_accumulate, :7913).  All
// gradients are holomorphic: for a real loss L of complex z, G = dL/dz with
// dL = Re(sum G dz).
// ---------------------------------------------------------------------------

// gbv[b, label[c], j, m_idx[t, j]] += gout[b, c] coeff[t] prod_{j' != j} bv[b, label[c], j', m_idx[t, j']]
void yo_factorized_schedule_adjoint(const void* bv_in, i64 batch, i64 basis, i64 blocks, i64 mdim,
                                    const i64* off, const i64* labels, const i64* midx, const void* coeffs_in,
                                    i64 comps, const void* gout_in, void* gbv_out, int threads) {
  const c128* bv = static_cast<const c128*>(bv_in);
  const c128* coeffs = static_cast<const c128*>(coeffs_in);
  const c128* gout = static_cast<const c128*>(gout_in);
  c128* gbv = static_cast<c128*>(gbv_out);
  parallel_chunks(batch, threads, [&](i64 lo, i64 hi) {
    std::vector<c128> f(blocks);
    for (i64 b = lo; b < hi; ++b) {
      for (i64 c = 0; c < comps; ++c) {
        const c128 g = gout[b * comps + c];
        if (g == c128(0, 0)) continue;
        const c128* row = bv + (b * basis + labels[c]) * blocks * mdim;
        c128* grow = gbv + (b * basis + labels[c]) * blocks * mdim;
        for (i64 t = off[c]; t < off[c + 1]; ++t) {
          for (i64 j = 0; j < blocks; ++j) f[j] = row[j * mdim + midx[t * blocks + j]];
          for (i64 j = 0; j < blocks; ++j) {
            c128 p = g * coeffs[t];
            for (i64 k = 0; k < blocks; ++k)
              if (k != j) p *= f[k];
            grow[j * mdim + midx[t * blocks + j]] += p;
          }
        }
      }
    }
  });
}

// Adjoint of out[b, o] = sum_{t in [off[o], off[o+1])} val[t] prod_i x[b, i]^{k[t, i]}:
//   gx[b, i] += gout[b, o] val[t] k[t, i] x_i^{k[t, i] - 1} prod_{i' != i} x_{i'}^{k[t, i']}
void yo_symmetric_power_monomial_adjoint(const void* x_in, i64 batch, i64 in_dim, const i64* counts,
                                         const i64* offsets, const void* values_in, i64 out_dim,
                                         const void* gout_in, void* gx_out) {
  const c128* x = static_cast<const c128*>(x_in);
  const c128* values = static_cast<const c128*>(values_in);
  const c128* gout = static_cast<const c128*>(gout_in);
  c128* gx = static_cast<c128*>(gx_out);
  for (i64 b = 0; b < batch; ++b) {
    const c128* xb = x + b * in_dim;
    for (i64 o = 0; o < out_dim; ++o) {
      const c128 g = gout[b * out_dim + o];
      if (g == c128(0, 0)) continue;
      for (i64 t = offsets[o]; t < offsets[o + 1]; ++t) {
        const i64* kt = counts + t * in_dim;
        for (i64 i = 0; i < in_dim; ++i) {
          if (kt[i] == 0) continue;
          c128 p = g * values[t] * double(kt[i]);
          for (i64 i2 = 0; i2 < in_dim; ++i2) {
            const i64 pw = kt[i2] - (i2 == i ? 1 : 0);
            for (i64 q = 0; q < pw; ++q) p *= xb[i2];
          }
          gx[b * in_dim + i] += p;
        }
      }
    }
  }
}

// g_e = dE_i / dd_e for every edge e = (i -> nbr[e]) of the rows, from the
// holomorphic G = dE/dA of the density above:
//   dA[n, lm] = p (R'_n(r) (d/r) Yc_lm + R_n grad Yc_lm) . dd
//   g_e = p Re( sum_{n, lm} G[n, lm] (R'_n (d/r) Yc_lm + R_n grad Yc_lm) )
void yo_ace_edge_grad(const double* disp, const i64* row_off, const int* nbr, const int* species,
                      const double* prefactor, i64 N, i64 nmax, i64 lmax, double rc, double lam,
                      const double* G_in /* complex128 [N, nmax, W] */, double* g /* [E, 3] */) {
  const i64 W = (lmax + 1) * (lmax + 1);
  const c128* G = reinterpret_cast<const c128*>(G_in);
  std::vector<double> rv(nmax + 1), rd(nmax + 1);
  std::vector<c128> yv(W), yd(3 * W);
  for (i64 i = 0; i < N; ++i) {
    const c128* Gi = G + i * nmax * W;
    for (i64 e = row_off[i]; e < row_off[i + 1]; ++e) {
      const double* d = disp + 3 * e;
      const double r = std::sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
      radial_one<double>(r, rc, lam, nmax, rv.data(), rd.data());
      sh_table<double>(d, 1, lmax, false, 1e-12, yv.data(), yd.data());
      const double p = prefactor[species[nbr[e]]];
      const double sr = std::max(r, 1e-12);
      double acc[3] = {0.0, 0.0, 0.0};
      for (i64 n = 1; n <= nmax; ++n) {
        for (i64 k = 0; k < W; ++k) {
          const c128 gk = Gi[(n - 1) * W + k];
          for (int a = 0; a < 3; ++a) {
            const c128 dA = rd[n] * (d[a] / sr) * yv[k] + rv[n] * yd[3 * k + a];
            acc[a] += (gk * dA).real();
          }
        }
      }
      for (int a = 0; a < 3; ++a) g[3 * e + a] = p * acc[a];
    }
  }
}

// F_k = -dE/dr_k = sum_{e in row k} g_e - sum_{e : nbr[e] = k} g_e  (d_e = r_nbr - r_row)
void yo_forces_from_edges(const i64* row_off, const int* nbr, i64 N, const double* g, double* F) {
  std::fill(F, F + 3 * N, 0.0);
  for (i64 i = 0; i < N; ++i)
    for (i64 e = row_off[i]; e < row_off[i + 1]; ++e)
      for (int a = 0; a < 3; ++a) {
        F[3 * i + a] += g[3 * e + a];
        F[3 * nbr[e] + a] -= g[3 * e + a];
      }
}

// ---------------------------------------------------------------------------
// Radial channel mixing (pace_radial_channel_contraction_with_derivative,
// ye3t/runtime/csrc/ye3t_runtime_core.cpp:651): out[p, o] = sum_i W[o, i] in[p, i]
// and the same for the derivatives, inputs in order, multiply then add.
// ---------------------------------------------------------------------------
void yo_radial_channel_contraction(int dtype, const void* in, const void* din, const void* W, i64 P, i64 I, i64 O,
                                   void* out, void* dout) {
  if (dtype == 0)
    contraction<float>(static_cast<const float*>(in), static_cast<const float*>(din),
                       static_cast<const float*>(W), P, I, O, static_cast<float*>(out), static_cast<float*>(dout));
  else
    contraction<double>(static_cast<const double*>(in), static_cast<const double*>(din),
                        static_cast<const double*>(W), P, I, O, static_cast<double*>(out),
                        static_cast<double*>(dout));
}

// A-basis with channels mixed per species pair (fp64): the composition of the
// radial table (execution_plan.py:7298, indices 1..nmax), the contraction
// above with the table W[z_i, z_j] (row-major [channel][n]), the complex
// harmonics (:7479) and density_accumulate (:7913), edges in CSR order:
//   A[i, c, lm] = sum_{e in row i} Rm_c(e) Yc_lm(d_e),  Rm_c = sum_n W[z_i, z_j, c, n-1] R_n(r)
void yo_ace_density_mixed(const double* disp, const i64* row_off, const int* nbr, const int* species,
                          const double* mixing, i64 N, i64 S, i64 C, i64 nmax, i64 lmax, double rc, double lam,
                          double* A_out /* complex128 [N, C, (lmax+1)^2] */) {
  const i64 W = (lmax + 1) * (lmax + 1);
  c128* A = reinterpret_cast<c128*>(A_out);
  std::vector<double> rv(nmax + 1), rd(nmax + 1), rm(C), dm(C);
  std::vector<c128> yv(W), yd(3 * W);
  for (i64 i = 0; i < N; ++i) {
    c128* Ai = A + i * C * W;
    for (i64 k = 0; k < C * W; ++k) Ai[k] = c128(0, 0);
    for (i64 e = row_off[i]; e < row_off[i + 1]; ++e) {
      const double* d = disp + 3 * e;
      const double r = std::sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2]);
      radial_one<double>(r, rc, lam, nmax, rv.data(), rd.data());
      const double* Wp = mixing + (i64(species[i]) * S + species[nbr[e]]) * C * nmax;
      contraction<double>(rv.data() + 1, rd.data() + 1, Wp, 1, nmax, C, rm.data(), dm.data());
      sh_table<double>(d, 1, lmax, false, 1e-12, yv.data(), yd.data());
      for (i64 c = 0; c < C; ++c)
        for (i64 k = 0; k < W; ++k) Ai[c * W + k] += rm[c] * yv[k];
    }
  }
}

}  // extern "C"
