// Per-edge radial and spherical-harmonic math shared by the standalone
// table kernels (edge_tables.cu) and the fused A-basis kernel (ace.cu).
#pragma once

#include <cmath>

#include "common.cuh"

namespace y3b {

constexpr int kMaxL = 10;                                  // harmonics degree limit
constexpr int kNormCount = (kMaxL + 1) * (kMaxL + 2) / 2;  // (l, m >= 0) pairs

// Orthonormal Condon-Shortley normalisation N_lm (m >= 0), passed to kernels
// by value.  Filled on the host with the formula of
// ye3t/core/spherical.py:66-77:
//   N_lm = exp((log(2l+1) - log(4 pi) + lgamma(l-m+1) - lgamma(l+m+1)) / 2)
struct ShNorm {
  double n[kNormCount];
};

__host__ __device__ __forceinline__ int norm_index(int l, int m) { return l * (l + 1) / 2 + m; }

inline ShNorm make_sh_norm() {
  ShNorm t;
  for (int l = 0; l <= kMaxL; ++l)
    for (int m = 0; m <= l; ++m)
      t.n[norm_index(l, m)] = std::exp(0.5 * (std::log(2.0 * l + 1.0) - std::log(4.0 * M_PI) +
                                              std::lgamma(double(l - m + 1)) -
                                              std::lgamma(double(l + m + 1))));
  return t;
}

// ChebExpCos radial basis k = 0..kmax with d/dr (ye3t_runtime_core.cpp:320-392):
//   s = r / max(rc, eps), zero beyond s > 1;  R_0 = 1;  R_1 = (1 + cos(pi s))/2;
//   R_k = (1 - T_k(x)) (1 + cos(pi s)) / 4,  x = 1 - 2 expm1(-lam (s-1)) / expm1(lam).
// The CUDA cos/sin/exp/expm1 functions are called as they are.
template <typename R>
__device__ __forceinline__ void radial_basis(R r, R rc_in, R lam, int kmax, R* val, R* der) {
  const R pi = R(3.141592653589793238462643383279502884);
  const R eps = sizeof(R) == 8 ? R(2.220446049250313e-16) : R(1.1920929e-07);
  const R rc = rc_in > eps ? rc_in : eps;
  const R s = r / rc;
#pragma unroll
  for (int k = 0; k <= kmax; ++k) {
    val[k] = R(0);
    if (der) der[k] = R(0);
  }
  if (s > R(1)) return;
  val[0] = R(1);
  R sn, cs;
  if (sizeof(R) == 8) {
    double sd, cd;
    sincos(double(pi * s), &sd, &cd);
    sn = R(sd); cs = R(cd);
  } else {
    float sf, cf;
    sincosf(float(pi * s), &sf, &cf);
    sn = R(sf); cs = R(cf);
  }
  const R env = R(1) + cs;
  const R denv = -pi * sn / rc;
  if (kmax >= 1) {
    val[1] = R(0.5) * env;
    if (der) der[1] = R(0.5) * denv;
  }
  if (kmax < 2) return;
  const R arg = -lam * (s - R(1));
  const R em = expm1(arg);
  const R den = expm1(lam);
  const R x = R(1) - R(2) * em / den;
  const R dx = R(2) * lam * exp(arg) / (den * rc);
  R t0 = R(1), t1 = x, u0 = R(1), u1 = R(2) * x;
#pragma unroll
  for (int k = 2; k <= kmax; ++k) {
    const R t2 = R(2) * x * t1 - t0;
    t0 = t1;
    t1 = t2;
    val[k] = R(0.25) * (R(1) - t1) * env;
    if (der) der[k] = R(0.25) * (-(R(k) * u1) * dx * env + (R(1) - t1) * denv);
    const R u2 = R(2) * x * u1 - u0;
    u0 = u1;
    u1 = u2;
  }
}

// Q_l^m(z) = d^m P_l(z)/dz^m for 0 <= m <= l <= LMAX via the fixed-m
// recurrence  Q_m^m = (2m-1)!!,  Q_{m+1}^m = (2m+1) z Q_m^m,
//   (l-m) Q_l^m = (2l-1) z Q_{l-1}^m - (l+m-1) Q_{l-2}^m,
// stored at q[norm_index(l, m)].  dQ_l^m/dz = Q_l^{m+1} (zero for m = l).
template <typename R, int LMAX>
__device__ __forceinline__ void legendre_derivs(R z, R* q) {
  R dfact = R(1);
#pragma unroll
  for (int m = 0; m <= LMAX; ++m) {
    if (m > 0) dfact *= R(2 * m - 1);
    R qa = dfact;
    q[norm_index(m, m)] = qa;
    if (m + 1 <= LMAX) {
      R qb = R(2 * m + 1) * z * qa;
      q[norm_index(m + 1, m)] = qb;
#pragma unroll
      for (int l = m + 2; l <= LMAX; ++l) {
        const R qc = (R(2 * l - 1) * z * qb - R(l + m - 1) * qa) / R(l - m);
        q[norm_index(l, m)] = qc;
        qa = qb;
        qb = qc;
      }
    }
  }
}

// The per-edge state of the real tesseral harmonics below: the Legendre
// derivative table and the powers (ux + i uy)^m.  real_sh_pair turns it into
// the values and gradients of the pair (l, +m), (l, -m) with the same
// arithmetic as real_sh_unit, so that a caller can form one pair at a time.
template <typename R, int LMAX>
struct ShState {
  R q[(LMAX + 1) * (LMAX + 2) / 2];
  R pr[LMAX + 1], pi_[LMAX + 1];
};

template <typename R, int LMAX>
__device__ __forceinline__ void sh_state(R ux, R uy, R uz, ShState<R, LMAX>& st) {
  legendre_derivs<R, LMAX>(uz, st.q);
  st.pr[0] = R(1);
  st.pi_[0] = R(0);
#pragma unroll
  for (int m = 1; m <= LMAX; ++m) {
    st.pr[m] = st.pr[m - 1] * ux - st.pi_[m - 1] * uy;
    st.pi_[m] = st.pr[m - 1] * uy + st.pi_[m - 1] * ux;
  }
}

// Values and polynomial gradients of (l, +m) [index 0] and (l, -m) [index 1]
// (for m = 0 only index 0 is set).
template <typename R, int LMAX>
__device__ __forceinline__ void real_sh_pair(int l, int m, const ShState<R, LMAX>& st, const ShNorm& nrm, R v[2],
                                             R g[2][3]) {
  const R rt2 = R(1.4142135623730950488016887242096981);
  if (m == 0) {
    const R n0 = R(nrm.n[norm_index(l, 0)]);
    v[0] = n0 * st.q[norm_index(l, 0)];
    g[0][0] = R(0);
    g[0][1] = R(0);
    g[0][2] = l >= 1 ? n0 * st.q[norm_index(l, 1)] : R(0);
    return;
  }
  const R sc = rt2 * R(nrm.n[norm_index(l, m)]);
  const R qq = st.q[norm_index(l, m)];
  const R dq = (m + 1 <= l) ? st.q[norm_index(l, m + 1)] : R(0);
  const R mr = R(m) * st.pr[m - 1], mi = R(m) * st.pi_[m - 1];
  v[0] = sc * qq * st.pr[m];
  v[1] = -sc * qq * st.pi_[m];
  g[0][0] = sc * qq * mr;
  g[0][1] = sc * qq * (-mi);
  g[0][2] = sc * dq * st.pr[m];
  g[1][0] = -sc * qq * mi;
  g[1][1] = -sc * qq * mr;
  g[1][2] = -sc * dq * st.pi_[m];
}

// Real tesseral harmonics (ye3t_runtime_core.cpp:226-290 convention) for all
// l <= LMAX at a unit vector u, with the gradient g[.][3] of their polynomial
// extension in (ux, uy, uz) when g != nullptr.  Packed columns [l^2, (l+1)^2).
template <typename R, int LMAX>
__device__ __forceinline__ void real_sh_unit(R ux, R uy, R uz, const ShNorm& nrm, R* v, R (*g)[3]) {
  R q[(LMAX + 1) * (LMAX + 2) / 2];
  legendre_derivs<R, LMAX>(uz, q);
  const R rt2 = R(1.4142135623730950488016887242096981);
  R pr[LMAX + 1], pi_[LMAX + 1];  // (ux + i uy)^m
  pr[0] = R(1);
  pi_[0] = R(0);
#pragma unroll
  for (int m = 1; m <= LMAX; ++m) {
    pr[m] = pr[m - 1] * ux - pi_[m - 1] * uy;
    pi_[m] = pr[m - 1] * uy + pi_[m - 1] * ux;
  }
#pragma unroll
  for (int l = 0; l <= LMAX; ++l) {
    const int c = l * l + l;
    const R n0 = R(nrm.n[norm_index(l, 0)]);
    v[c] = n0 * q[norm_index(l, 0)];
    if (g) {
      g[c][0] = R(0);
      g[c][1] = R(0);
      g[c][2] = l >= 1 ? n0 * q[norm_index(l, 1)] : R(0);
    }
#pragma unroll
    for (int m = 1; m <= l; ++m) {
      const R sc = rt2 * R(nrm.n[norm_index(l, m)]);
      const R qq = q[norm_index(l, m)];
      const R dq = (m + 1 <= l) ? q[norm_index(l, m + 1)] : R(0);
      v[c + m] = sc * qq * pr[m];
      v[c - m] = -sc * qq * pi_[m];
      if (g) {
        const R mr = R(m) * pr[m - 1], mi = R(m) * pi_[m - 1];
        g[c + m][0] = sc * qq * mr;
        g[c + m][1] = sc * qq * (-mi);
        g[c + m][2] = sc * dq * pr[m];
        g[c - m][0] = -sc * qq * mi;
        g[c - m][1] = -sc * qq * mr;
        g[c - m][2] = -sc * dq * pi_[m];
      }
    }
  }
}

}  // namespace y3b
