// Standalone radial and spherical-harmonic table kernels (one thread per edge).
#include "edge_math.cuh"

namespace y3b {

constexpr int kMaxRadial = 64;

template <typename R>
__global__ void __launch_bounds__(128) radial_table_kernel(const R* __restrict__ radii,
                                                           const R* __restrict__ cutoffs,
                                                           const R* __restrict__ lambdas, int64_t E,
                                                           int kmax, R* __restrict__ val,
                                                           R* __restrict__ der) {
  R v[kMaxRadial + 1], d[kMaxRadial + 1];
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < E;
       e += int64_t(gridDim.x) * blockDim.x) {
    radial_basis<R>(radii[e], cutoffs[e], lambdas[e], kmax, v, d);
    for (int k = 0; k <= kmax; ++k) {
      val[e * (kmax + 1) + k] = v[k];
      der[e * (kmax + 1) + k] = d[k];
    }
  }
}

// Cartesian derivative of a unit-sphere function through u = r / max(|r|, eps):
// J = (I - u u^T) / |r| above eps, I / eps below (ye3t_runtime_core.cpp:819-834).
template <typename R, int LMAX, bool COMPLEX>
__global__ void __launch_bounds__(128) sh_table_kernel(const R* __restrict__ vec, int64_t E, R eps,
                                                       ShNorm nrm, R* __restrict__ val,
                                                       R* __restrict__ der) {
  constexpr int W = (LMAX + 1) * (LMAX + 1);
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < E;
       e += int64_t(gridDim.x) * blockDim.x) {
    const R x = vec[3 * e], y = vec[3 * e + 1], z = vec[3 * e + 2];
    const R r = sqrt(x * x + y * y + z * z);
    const R sr = r > eps ? r : eps;
    const R u[3] = {x / sr, y / sr, z / sr};
    R jac[3][3];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b)
        jac[a][b] = (r > eps) ? ((a == b ? R(1) : R(0)) - u[a] * u[b]) / sr
                              : (a == b ? R(1) / sr : R(0));
    R v[W], g[W][3];
    real_sh_unit<R, LMAX>(u[0], u[1], u[2], nrm, v, g);
    R d[W][3];
#pragma unroll
    for (int i = 0; i < W; ++i)
#pragma unroll
      for (int a = 0; a < 3; ++a) d[i][a] = g[i][0] * jac[a][0] + g[i][1] * jac[a][1] + g[i][2] * jac[a][2];
    if (!COMPLEX) {
#pragma unroll
      for (int i = 0; i < W; ++i) {
        val[e * W + i] = v[i];
#pragma unroll
        for (int a = 0; a < 3; ++a) der[(e * W + i) * 3 + a] = d[i][a];
      }
    } else {
      // Complex Condon-Shortley from the real table (ye3t_runtime_core.cpp:891-948):
      //   Yc_{l,-m} = (R_{+m} + i R_{-m}) / sqrt2,  Yc_{l,+m} = (-1)^m (R_{+m} - i R_{-m}) / sqrt2.
      const R inv2 = R(0.70710678118654752440084436210484903);
#pragma unroll
      for (int l = 0; l <= LMAX; ++l) {
        const int c = l * l + l;
        val[2 * (e * W + c)] = v[c];
        val[2 * (e * W + c) + 1] = R(0);
#pragma unroll
        for (int a = 0; a < 3; ++a) {
          der[2 * ((e * W + c) * 3 + a)] = d[c][a];
          der[2 * ((e * W + c) * 3 + a) + 1] = R(0);
        }
#pragma unroll
        for (int m = 1; m <= l; ++m) {
          const R sg = (m & 1) ? R(-1) : R(1);
          const int p = c + m, n = c - m;
          val[2 * (e * W + n)] = inv2 * v[p];
          val[2 * (e * W + n) + 1] = inv2 * v[n];
          val[2 * (e * W + p)] = sg * (inv2 * v[p]);
          val[2 * (e * W + p) + 1] = sg * (inv2 * -v[n]);
#pragma unroll
          for (int a = 0; a < 3; ++a) {
            der[2 * ((e * W + n) * 3 + a)] = inv2 * d[p][a];
            der[2 * ((e * W + n) * 3 + a) + 1] = inv2 * d[n][a];
            der[2 * ((e * W + p) * 3 + a)] = sg * (inv2 * d[p][a]);
            der[2 * ((e * W + p) * 3 + a) + 1] = sg * (inv2 * -d[n][a]);
          }
        }
      }
    }
  }
}

template <typename R, int LMAX>
int launch_sh(const R* vec, int64_t E, R eps, bool complex_out, R* val, R* der, cudaStream_t s) {
  const int threads = 128;
  const int grid = grid_for(E, threads);
  const ShNorm nrm = make_sh_norm();
  if (complex_out)
    sh_table_kernel<R, LMAX, true><<<grid, threads, 0, s>>>(vec, E, eps, nrm, val, der);
  else
    sh_table_kernel<R, LMAX, false><<<grid, threads, 0, s>>>(vec, E, eps, nrm, val, der);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

template <typename R>
int dispatch_sh(const R* vec, int64_t E, int lmax, R eps, bool complex_out, R* val, R* der,
                cudaStream_t s) {
  switch (lmax) {
    case 0: return launch_sh<R, 0>(vec, E, eps, complex_out, val, der, s);
    case 1: return launch_sh<R, 1>(vec, E, eps, complex_out, val, der, s);
    case 2: return launch_sh<R, 2>(vec, E, eps, complex_out, val, der, s);
    case 3: return launch_sh<R, 3>(vec, E, eps, complex_out, val, der, s);
    case 4: return launch_sh<R, 4>(vec, E, eps, complex_out, val, der, s);
    case 5: return launch_sh<R, 5>(vec, E, eps, complex_out, val, der, s);
    case 6: return launch_sh<R, 6>(vec, E, eps, complex_out, val, der, s);
    case 7: return launch_sh<R, 7>(vec, E, eps, complex_out, val, der, s);
    case 8: return launch_sh<R, 8>(vec, E, eps, complex_out, val, der, s);
    default: return fail(Y3B_ERR_UNSUPPORTED, "spherical harmonics: lmax %d > 8 not built", lmax);
  }
}

}  // namespace y3b

using namespace y3b;

extern "C" int y3b_cheb_exp_cos_radial_table(int dtype, const void* radii, const void* cutoffs,
                                             const void* lambdas, int64_t edge_count,
                                             int64_t maximum_radial_index, void* values,
                                             void* derivatives, void* stream) {
  Y3B_CHECK_ARG(edge_count >= 0, "negative edge count");
  Y3B_CHECK_ARG(maximum_radial_index >= 0 && maximum_radial_index <= kMaxRadial,
                "maximum_radial_index must be in [0, %d]", kMaxRadial);
  if (edge_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(radii && cutoffs && lambdas && values && derivatives, "null pointer argument");
  const int threads = 128;
  const int grid = grid_for(edge_count, threads);
  Y3B_DISPATCH_REAL(dtype, R, {
    radial_table_kernel<R><<<grid, threads, 0, as_stream(stream)>>>(
        static_cast<const R*>(radii), static_cast<const R*>(cutoffs),
        static_cast<const R*>(lambdas), edge_count, int(maximum_radial_index),
        static_cast<R*>(values), static_cast<R*>(derivatives));
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_spherical_harmonics_table(int dtype, const void* edge_vectors, int64_t edge_count,
                                             int64_t maximum_angular_momentum, int real_output,
                                             double epsilon, void* values, void* derivatives,
                                             void* stream) {
  Y3B_CHECK_ARG(edge_count >= 0, "negative edge count");
  Y3B_CHECK_ARG(maximum_angular_momentum >= 0, "negative maximum_angular_momentum");
  if (edge_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(edge_vectors && values && derivatives, "null pointer argument");
  const bool cplx = real_output == 0;
  if (dtype == Y3B_F64)
    return dispatch_sh<double>(static_cast<const double*>(edge_vectors), edge_count,
                               int(maximum_angular_momentum), epsilon, cplx,
                               static_cast<double*>(values), static_cast<double*>(derivatives),
                               as_stream(stream));
  if (dtype == Y3B_F32)
    return dispatch_sh<float>(static_cast<const float*>(edge_vectors), edge_count,
                              int(maximum_angular_momentum), float(epsilon), cplx,
                              static_cast<float*>(values), static_cast<float*>(derivatives),
                              as_stream(stream));
  return fail(Y3B_ERR_ARGUMENT, "spherical harmonics: dtype must be F32 or F64 (edge vectors)");
}
