// Radial channel mixing.
//
//  * y3b_radial_channel_contraction: out[p, o] = sum_i W[o, i] in[p, i] and the
//    same for the radial derivatives, as pace_radial_channel_contraction_with_
//    derivative (ye3t/runtime/csrc/ye3t_runtime_core.cpp:651).
//  * y3b_ace_density_mixed: the A-basis with channels mixed per species pair,
//      A[i, c, l^2 + l + m] = sum_{j in row i} Rm_c(z_i, z_j, r_ij) Yc_lm(r_ij),
//      Rm_c = sum_n W[z_i, z_j, c, n] R_n(r),  n = 1..nmax,
//    the composition of the ChebExpCos table (execution_plan.py:7298), the
//    contraction above applied with the pair's table, the complex harmonics
//    (:7479) and density_accumulate (:7913), fused: one warp per centre, no
//    atomics, every A row written once.
#include "common.cuh"
#include "edge_math.cuh"
#include "neighbors.cuh"

namespace y3b {

namespace {

// Separate multiply and add (no contraction), as the reference's loop.
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }

template <typename T>
__global__ void radial_contraction_kernel(const T* __restrict__ in, const T* __restrict__ din,
                                          const T* __restrict__ W, int64_t P, int64_t I, int64_t O,
                                          T* __restrict__ out, T* __restrict__ dout) {
  const int64_t total = P * O;
  for (int64_t q = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; q < total;
       q += int64_t(gridDim.x) * blockDim.x) {
    const int64_t p = q / O, o = q - p * O;
    const T* x = in + p * I;
    const T* dx = din + p * I;
    const T* w = W + o * I;
    T v = T(0), d = T(0);
    for (int64_t i = 0; i < I; ++i) {
      const T c = __ldg(w + i);
      v = add_rn(v, mul_rn(c, x[i]));
      d = add_rn(d, mul_rn(c, dx[i]));
    }
    out[q] = v;
    dout[q] = d;
  }
}

template <typename T> struct Cx;
template <> struct Cx<float> { using type = float2; };
template <> struct Cx<double> { using type = double2; };

__device__ __forceinline__ float2 mk(float x, float y) { return make_float2(x, y); }
__device__ __forceinline__ double2 mk(double x, double y) { return make_double2(x, y); }

constexpr int kMaxRadial = 16;  // radial indices 1..nmax
constexpr int kMixWarps = 4;
constexpr int kMixOut = 8;  // outputs per lane per pass

// One warp per centre.  Pass 1: lanes over up to 32 edges form the mixed radial
// channels Rm_c and the complex harmonics into warp-private shared memory.
// Pass 2: lanes over the C*(lmax+1)^2 outputs, kMixOut at a time, sum those
// edges in CSR order; rows longer than 32 edges add their later chunks to the
// A row this warp owns.
template <typename T, int LMAX>
__global__ void __launch_bounds__(32 * kMixWarps) ace_density_mixed_kernel(
    const double* __restrict__ pos, const int32_t* __restrict__ species, int64_t N, int64_t center_begin,
    int64_t count, double box, const int64_t* __restrict__ row_off, const int32_t* __restrict__ nbr,
    const T* __restrict__ mix, int S, int C, int nmax, T rc, T lam, ShNorm nrm,
    typename Cx<T>::type* __restrict__ A, int32_t* status) {
  using C2 = typename Cx<T>::type;
  constexpr int W = (LMAX + 1) * (LMAX + 1);
  extern __shared__ __align__(16) unsigned char msm[];
  // pair tables one element apart, so lanes reading the tables of different
  // neighbour species hit different banks
  const int pstride = C * nmax + 1;
  const int mixn = S * S * pstride;
  T* s_mix = reinterpret_cast<T*>(msm);
  C2* s_y = reinterpret_cast<C2*>(msm + ((size_t(mixn) * sizeof(T) + 15) & ~size_t(15)));  // [warp][32][W]
  T* s_rm = reinterpret_cast<T*>(s_y + kMixWarps * 32 * W);                                   // [warp][32][C]
  for (int k = threadIdx.x; k < S * S * C * nmax; k += blockDim.x) {
    const int pr = k / (C * nmax);
    s_mix[pr * pstride + (k - pr * C * nmax)] = mix[k];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  C2* y_w = s_y + wib * 32 * W;
  T* rm_w = s_rm + wib * 32 * C;
  const int nout = C * W;
  const int64_t row0 = row_off[0];
  for (int64_t a = blockIdx.x * int64_t(kMixWarps) + wib; a < count; a += int64_t(gridDim.x) * kMixWarps) {
    const int64_t i = center_begin + a;
    int zi = species[i];
    if (zi < 0 || zi >= S) {
      if (status && lane == 0) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
      zi = -1;
    }
    const int64_t b = row_off[a] - row0, e = row_off[a + 1] - row0;
    C2* Ai = A + a * int64_t(nout);
    bool first = true;
    for (int64_t c0 = b; c0 < e || first; c0 += 32) {
      const int nedge = c0 < e ? ((e - c0) < 32 ? int(e - c0) : 32) : 0;
      if (lane < nedge) {
        const int64_t j = nbr[c0 + lane];
        const int zj = (j >= 0 && j < N) ? species[j] : -1;
        if (j < 0 || j >= N || zj < 0 || zj >= S || zi < 0) {
          if (status && (j < 0 || j >= N || zj < 0 || zj >= S)) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
          for (int c = 0; c < C; ++c) rm_w[lane * C + c] = T(0);
#pragma unroll
          for (int k = 0; k < W; ++k) y_w[lane * W + k] = mk(T(0), T(0));
        } else {
          double dd[3];
          min_image(pos, i, j, box, dd);
          const double r2 = dist2(dd);
          const T d[3] = {T(dd[0]), T(dd[1]), T(dd[2])};
          const T r = sqrt(T(r2));
          T rv[kMaxRadial + 1];
          radial_basis<T>(r, rc, lam, nmax, rv, nullptr);
          const T* wp = s_mix + (size_t(zi) * S + zj) * pstride;
          for (int c = 0; c < C; ++c) {
            T s = T(0);
            for (int n = 0; n < nmax; ++n) s = add_rn(s, mul_rn(wp[c * nmax + n], rv[n + 1]));
            rm_w[lane * C + c] = s;
          }
          const T sr = r > T(1e-12) ? r : T(1e-12);
          T v[W];
          real_sh_unit<T, LMAX>(d[0] / sr, d[1] / sr, d[2] / sr, nrm, v, nullptr);
          const T inv2 = T(0.70710678118654752440084436210484903);
#pragma unroll
          for (int l = 0; l <= LMAX; ++l) {
            const int cc = l * l + l;
            y_w[lane * W + cc] = mk(v[cc], T(0));
#pragma unroll
            for (int m = 1; m <= l; ++m) {
              const T sg = (m & 1) ? T(-1) : T(1);
              y_w[lane * W + cc - m] = mk(inv2 * v[cc + m], inv2 * v[cc - m]);
              y_w[lane * W + cc + m] = mk(sg * (inv2 * v[cc + m]), sg * (inv2 * -v[cc - m]));
            }
          }
        }
      }
      __syncwarp();
      for (int o0 = 0; o0 < nout; o0 += 32 * kMixOut) {
        C2 acc[kMixOut];
#pragma unroll
        for (int k = 0; k < kMixOut; ++k) acc[k] = mk(T(0), T(0));
        for (int q = 0; q < nedge; ++q) {
#pragma unroll
          for (int k = 0; k < kMixOut; ++k) {
            const int o = o0 + lane + 32 * k;
            if (o < nout) {
              const int c = o / W, lm = o - c * W;
              const T rp = rm_w[q * C + c];
              const C2 y = y_w[q * W + lm];
              acc[k].x += rp * y.x;
              acc[k].y += rp * y.y;
            }
          }
        }
#pragma unroll
        for (int k = 0; k < kMixOut; ++k) {
          const int o = o0 + lane + 32 * k;
          if (o < nout) {
            if (first) Ai[o] = acc[k];
            else Ai[o] = mk(Ai[o].x + acc[k].x, Ai[o].y + acc[k].y);
          }
        }
      }
      first = false;
      __syncwarp();
    }
  }
}

}  // namespace
}  // namespace y3b

using namespace y3b;

extern "C" int y3b_radial_channel_contraction(int dtype, const void* input_values, const void* input_derivatives,
                                              const void* coefficients, int64_t point_count, int64_t input_count,
                                              int64_t output_count, void* output_values, void* output_derivatives,
                                              void* stream) {
  Y3B_CHECK_ARG(point_count >= 0 && input_count > 0 && output_count > 0,
                "invalid radial contraction dimensions");
  if (point_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(input_values && input_derivatives && coefficients && output_values && output_derivatives,
                "radial contraction received a null array");
  const int grid = grid_for(point_count * output_count, 256);
  cudaStream_t s = as_stream(stream);
  Y3B_DISPATCH_REAL(dtype, T,
                    radial_contraction_kernel<T><<<grid, 256, 0, s>>>(
                        static_cast<const T*>(input_values), static_cast<const T*>(input_derivatives),
                        static_cast<const T*>(coefficients), point_count, input_count, output_count,
                        static_cast<T*>(output_values), static_cast<T*>(output_derivatives)));
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_ace_density_mixed(int dtype, const double* positions, const int32_t* species, int64_t atom_count,
                                     int64_t center_begin, int64_t center_count, double box,
                                     const int64_t* row_offsets, const int32_t* neighbors, const void* mixing,
                                     int64_t species_count, int64_t channel_count, int64_t nmax, int64_t lmax,
                                     double cutoff, double lambda, void* A, int32_t* status, void* stream) {
  Y3B_CHECK_ARG(nmax >= 1 && nmax <= kMaxRadial, "nmax must be in [1, %d]", kMaxRadial);
  Y3B_CHECK_ARG(species_count >= 1 && channel_count >= 1 && channel_count <= 256, "bad species / channel count");
  Y3B_CHECK_ARG(center_begin >= 0 && center_count >= 0 && center_begin + center_count <= atom_count,
                "bad centre range");
  Y3B_CHECK_ARG(box > 0 && cutoff > 0, "box and cutoff must be positive");
  if (center_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(positions && species && row_offsets && mixing && A, "null pointer argument");
  const ShNorm nrm = make_sh_norm();
  const int S = int(species_count), C = int(channel_count);
  const int grid = int(std::min<int64_t>((center_count + kMixWarps - 1) / kMixWarps, int64_t(kSMs) * 32));
  cudaStream_t s = as_stream(stream);
  const size_t W = size_t(lmax + 1) * size_t(lmax + 1);
  auto smem_for = [&](size_t real_size) {
    return ((size_t(S) * S * (C * nmax + 1) * real_size + 15) & ~size_t(15)) + kMixWarps * 32 * W * 2 * real_size +
           kMixWarps * 32 * size_t(C) * real_size;
  };
#define Y3B_MIX_CASE(T, L)                                                                                    \
  case L: {                                                                                                   \
    const size_t smem = smem_for(sizeof(T));                                                                  \
    Y3B_CHECK_ARG(smem <= 200 * 1024, "mixing table and edge buffers need %zu bytes of shared memory", smem); \
    Y3B_CUDA_TRY(cudaFuncSetAttribute(ace_density_mixed_kernel<T, L>,                                         \
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));               \
    ace_density_mixed_kernel<T, L><<<grid, 32 * kMixWarps, smem, s>>>(                                        \
        positions, species, atom_count, center_begin, center_count, box, row_offsets, neighbors,              \
        static_cast<const T*>(mixing), S, C, int(nmax), T(cutoff), T(lambda), nrm,                           \
        static_cast<typename Cx<T>::type*>(A), status);                                                       \
    break;                                                                                                    \
  }
#define Y3B_MIX_L(T)                                                                            \
  switch (lmax) {                                                                               \
    Y3B_MIX_CASE(T, 0)                                                                          \
    Y3B_MIX_CASE(T, 1)                                                                          \
    Y3B_MIX_CASE(T, 2)                                                                          \
    Y3B_MIX_CASE(T, 3)                                                                          \
    Y3B_MIX_CASE(T, 4)                                                                          \
    default:                                                                                    \
      return fail(Y3B_ERR_UNSUPPORTED, "ace_density_mixed: lmax %lld not built (0..4)", (long long)lmax); \
  }
  if (dtype == Y3B_F32) {
    Y3B_MIX_L(float)
  } else if (dtype == Y3B_F64) {
    Y3B_MIX_L(double)
  } else {
    return fail(Y3B_ERR_ARGUMENT, "ace_density_mixed: dtype must be F32 or F64 (got %d)", dtype);
  }
#undef Y3B_MIX_L
#undef Y3B_MIX_CASE
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}
