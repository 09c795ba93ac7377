// Standalone edge-product operators of the runtime (the fused density kernels
// compute the same products in registers):
//  * scheduled radial x angular channels with their Cartesian derivatives
//    (scheduled_radial_angular_channels_with_derivative,
//    ye3t/runtime/execution_plan.py:7675, reference composition :7036-7080);
//  * the plain site-basis product with per-edge group prefactors, complex
//    capable (plain_site_basis_product_with_derivative, :7582, reference
//    composition :7082-7155), and its adjoint against edge-channel adjoints
//    (plain_site_basis_product_adjoint, :7790, composition :7158-7220).
// Each output entry is formed with the reference's operation order; the real
// operator rounds every product and sum separately (no contraction), as the
// reference's elementwise tensor operations do.
#include "common.cuh"

namespace y3b {

namespace {

__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

// values[e, c] = R[e, rad_c] Y[e, ang_c] s_c and derivatives[e, c, x] =
// s_c (R'[e, rad_c] d[e, x] Y[e, ang_c] + R[e, rad_c] dY[e, ang_c, x]) when
// channel_types[c] < 0 or equals edge_types[e], else 0.  One thread per
// (edge, channel); radial / angular indices outside their tables set
// Y3B_STATUS_INDEX_RANGE and give 0.
template <typename R>
__global__ void __launch_bounds__(256) scheduled_channels_kernel(
    const R* __restrict__ rv, const R* __restrict__ rd, int64_t K, const R* __restrict__ av,
    const R* __restrict__ ad, int64_t A, const R* __restrict__ dir, const int64_t* __restrict__ edge_types,
    int64_t E, const int64_t* __restrict__ crad, const int64_t* __restrict__ cang,
    const int64_t* __restrict__ ctype, const R* __restrict__ cscale, int64_t C, R* __restrict__ val,
    R* __restrict__ der, int32_t* __restrict__ status) {
  const int64_t total = E * C;
  for (int64_t lin = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; lin < total;
       lin += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = lin / C, c = lin - e * C;
    const int64_t k = __ldg(crad + c), a = __ldg(cang + c), ty = __ldg(ctype + c);
    R v = R(0), d[3] = {R(0), R(0), R(0)};
    if (k < 0 || k >= K || a < 0 || a >= A) {
      if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
    } else if (ty < 0 || ty == edge_types[e]) {
      const R s = __ldg(cscale + c);
      const R r = rv[e * K + k], r1 = rd[e * K + k], y = av[e * A + a];
      v = mul_rn(mul_rn(r, y), s);
#pragma unroll
      for (int x = 0; x < 3; ++x)
        d[x] = mul_rn(s, add_rn(mul_rn(mul_rn(r1, dir[3 * e + x]), y), mul_rn(r, ad[(e * A + a) * 3 + x])));
    }
    val[lin] = v;
#pragma unroll
    for (int x = 0; x < 3; ++x) der[3 * lin + x] = d[x];
  }
}

// Term t (group g = term_groups[t], channel ch = term_channels[t]) of edge e:
// values[e, ch] = p[g, e] R[g, e] Y[t, e], derivatives[e, ch, x] = p[g, e]
// (R'[g, e] d[e, x] Y[t, e] + R[g, e] dY[t, e, x]), and the prefactor
// derivative channels pc / pn [g, e] times R[g, e] Y[t, e].  One thread per
// (term, edge); the outputs start zeroed.  Out-of-range groups or channels set
// Y3B_STATUS_INDEX_RANGE and write nothing.
template <typename T>
__global__ void __launch_bounds__(256) plain_product_kernel(
    const T* __restrict__ rv, const T* __restrict__ rd, int64_t G, const T* __restrict__ av,
    const T* __restrict__ ad, int64_t Tn, const T* __restrict__ pref, const T* __restrict__ pc,
    const T* __restrict__ pn, const T* __restrict__ dir, int64_t E, const int64_t* __restrict__ groups,
    const int64_t* __restrict__ channels, int64_t C, T* __restrict__ val, T* __restrict__ der,
    T* __restrict__ charge_c, T* __restrict__ charge_n, int32_t* __restrict__ status) {
  const int64_t total = Tn * E;
  for (int64_t lin = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; lin < total;
       lin += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = lin / E, e = lin - t * E;
    const int64_t g = __ldg(groups + t), ch = __ldg(channels + t);
    if (g < 0 || g >= G || ch < 0 || ch >= C) {
      if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
      continue;
    }
    const T r = rv[g * E + e], r1 = rd[g * E + e], p = pref[g * E + e], y = av[t * E + e];
    const int64_t o = e * C + ch;
    val[o] = mul(mul(p, r), y);
#pragma unroll
    for (int x = 0; x < 3; ++x)
      der[3 * o + x] = mul(p, add(mul(mul(r1, dir[3 * e + x]), y), mul(r, ad[(t * E + e) * 3 + x])));
    const T common = mul(r, y);
    charge_c[o] = mul(pc[g * E + e], common);
    charge_n[o] = mul(pn[g * E + e], common);
  }
}

// Adjoint of the plain site-basis product with edge weights w[e] (and their
// Cartesian derivatives dw[e, :]) against edge-channel adjoints a[e, ch]
// (execution_plan.py:7790, composition :7158-7220): per edge,
//   position[e, :] = sum_t a[e, ch_t] (td[t, e, :] w[e] + tv[t, e] dw[e, :])
//   charge_center / neighbor[e] = sum_t a[e, ch_t] pc / pn[g_t, e] R[g_t, e] Y[t, e] w[e]
// with tv, td the term values and derivatives of the forward product.  One
// thread per edge, terms in order (no atomics).
template <typename T>
__global__ void __launch_bounds__(256) plain_product_adjoint_kernel(
    const T* __restrict__ rv, const T* __restrict__ rd, int64_t G, const T* __restrict__ av,
    const T* __restrict__ ad, int64_t Tn, const T* __restrict__ pref, const T* __restrict__ pc,
    const T* __restrict__ pn, const T* __restrict__ dir, const T* __restrict__ w, const T* __restrict__ dw,
    int64_t E, const int64_t* __restrict__ groups, const int64_t* __restrict__ channels, int64_t C,
    const T* __restrict__ adj, T* __restrict__ pos, T* __restrict__ charge_c, T* __restrict__ charge_n,
    int32_t* __restrict__ status) {
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < E; e += int64_t(gridDim.x) * blockDim.x) {
    T acc[3] = {zero<T>(), zero<T>(), zero<T>()}, cc = zero<T>(), cn = zero<T>();
    const T we = w[e];
    for (int64_t t = 0; t < Tn; ++t) {
      const int64_t g = __ldg(groups + t), ch = __ldg(channels + t);
      if (g < 0 || g >= G || ch < 0 || ch >= C) {
        if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
        continue;
      }
      const T r = rv[g * E + e], r1 = rd[g * E + e], p = pref[g * E + e], y = av[t * E + e];
      const T a = adj[e * C + ch];
      const T tv = mul(mul(p, r), y);
#pragma unroll
      for (int x = 0; x < 3; ++x) {
        const T td = mul(p, add(mul(mul(r1, dir[3 * e + x]), y), mul(r, ad[(t * E + e) * 3 + x])));
        acc[x] = add(acc[x], mul(a, add(mul(td, we), mul(tv, dw[3 * e + x]))));
      }
      const T common = mul(mul(r, y), we);
      cc = add(cc, mul(mul(a, pc[g * E + e]), common));
      cn = add(cn, mul(mul(a, pn[g * E + e]), common));
    }
#pragma unroll
    for (int x = 0; x < 3; ++x) pos[3 * e + x] = acc[x];
    charge_c[e] = cc;
    charge_n[e] = cn;
  }
}

}  // namespace
}  // namespace y3b

using namespace y3b;

extern "C" int y3b_scheduled_radial_angular_channels(
    int dtype, const void* radial_values, const void* radial_derivatives, int64_t radial_count,
    const void* angular_values, const void* angular_derivatives, int64_t angular_count,
    const void* radial_directions, const int64_t* edge_types, int64_t edge_count,
    const int64_t* channel_radial_indices, const int64_t* channel_angular_indices, const int64_t* channel_types,
    const void* channel_scales, int64_t channel_count, void* values, void* derivatives, int32_t* status,
    void* stream) {
  Y3B_CHECK_ARG(radial_count >= 0 && angular_count >= 0 && edge_count >= 0 && channel_count >= 0, "negative size");
  const int64_t total = edge_count * channel_count;
  if (total == 0) return Y3B_OK;
  Y3B_CHECK_ARG(radial_values && radial_derivatives && angular_values && angular_derivatives && radial_directions &&
                    edge_types && channel_radial_indices && channel_angular_indices && channel_types &&
                    channel_scales && values && derivatives,
                "null pointer argument");
  const int threads = 256;
  Y3B_DISPATCH_REAL(dtype, R, {
    scheduled_channels_kernel<R><<<grid_for(total, threads), threads, 0, as_stream(stream)>>>(
        static_cast<const R*>(radial_values), static_cast<const R*>(radial_derivatives), radial_count,
        static_cast<const R*>(angular_values), static_cast<const R*>(angular_derivatives), angular_count,
        static_cast<const R*>(radial_directions), edge_types, edge_count, channel_radial_indices,
        channel_angular_indices, channel_types, static_cast<const R*>(channel_scales), channel_count,
        static_cast<R*>(values), static_cast<R*>(derivatives), status);
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_plain_site_basis_product(
    int dtype, const void* radial_values, const void* radial_derivatives, int64_t group_count,
    const void* angular_values, const void* angular_derivatives, int64_t term_count, const void* prefactors,
    const void* prefactor_derivatives_center, const void* prefactor_derivatives_neighbor,
    const void* radial_directions, int64_t edge_count, const int64_t* term_groups, const int64_t* term_channels,
    int64_t channel_count, void* edge_values, void* edge_derivatives, void* charge_center, void* charge_neighbor,
    int32_t* status, void* stream) {
  Y3B_CHECK_ARG(group_count >= 0 && term_count >= 0 && edge_count >= 0 && channel_count >= 0, "negative size");
  if (edge_count == 0 || channel_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(edge_values && edge_derivatives && charge_center && charge_neighbor, "null output pointer");
  cudaStream_t s = as_stream(stream);
  size_t elem = 0;
  Y3B_DISPATCH(dtype, T, { elem = sizeof(T); });
  const size_t n = size_t(edge_count) * size_t(channel_count) * elem;
  Y3B_CUDA_TRY(cudaMemsetAsync(edge_values, 0, n, s));
  Y3B_CUDA_TRY(cudaMemsetAsync(edge_derivatives, 0, 3 * n, s));
  Y3B_CUDA_TRY(cudaMemsetAsync(charge_center, 0, n, s));
  Y3B_CUDA_TRY(cudaMemsetAsync(charge_neighbor, 0, n, s));
  const int64_t total = term_count * edge_count;
  if (total == 0) return Y3B_OK;
  Y3B_CHECK_ARG(radial_values && radial_derivatives && angular_values && angular_derivatives && prefactors &&
                    prefactor_derivatives_center && prefactor_derivatives_neighbor && radial_directions &&
                    term_groups && term_channels,
                "null pointer argument");
  const int threads = 256;
  Y3B_DISPATCH(dtype, T, {
    plain_product_kernel<T><<<grid_for(total, threads), threads, 0, s>>>(
        static_cast<const T*>(radial_values), static_cast<const T*>(radial_derivatives), group_count,
        static_cast<const T*>(angular_values), static_cast<const T*>(angular_derivatives), term_count,
        static_cast<const T*>(prefactors), static_cast<const T*>(prefactor_derivatives_center),
        static_cast<const T*>(prefactor_derivatives_neighbor), static_cast<const T*>(radial_directions),
        edge_count, term_groups, term_channels, channel_count, static_cast<T*>(edge_values),
        static_cast<T*>(edge_derivatives), static_cast<T*>(charge_center), static_cast<T*>(charge_neighbor),
        status);
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_plain_site_basis_product_adjoint(
    int dtype, const void* radial_values, const void* radial_derivatives, int64_t group_count,
    const void* angular_values, const void* angular_derivatives, int64_t term_count, const void* prefactors,
    const void* prefactor_derivatives_center, const void* prefactor_derivatives_neighbor,
    const void* radial_directions, const void* edge_weights, const void* edge_weight_derivatives, int64_t edge_count,
    const int64_t* term_groups, const int64_t* term_channels, int64_t channel_count, const void* edge_adjoint,
    void* position_adjoint, void* charge_center_adjoint, void* charge_neighbor_adjoint, int32_t* status,
    void* stream) {
  Y3B_CHECK_ARG(group_count >= 0 && term_count >= 0 && edge_count >= 0 && channel_count >= 0, "negative size");
  if (edge_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(edge_weights && edge_weight_derivatives && position_adjoint && charge_center_adjoint &&
                    charge_neighbor_adjoint && radial_directions &&
                    (term_count == 0 || (radial_values && radial_derivatives && angular_values &&
                                         angular_derivatives && prefactors && prefactor_derivatives_center &&
                                         prefactor_derivatives_neighbor && term_groups && term_channels &&
                                         edge_adjoint)),
                "null pointer argument");
  const int threads = 256;
  Y3B_DISPATCH(dtype, T, {
    plain_product_adjoint_kernel<T><<<grid_for(edge_count, threads), threads, 0, as_stream(stream)>>>(
        static_cast<const T*>(radial_values), static_cast<const T*>(radial_derivatives), group_count,
        static_cast<const T*>(angular_values), static_cast<const T*>(angular_derivatives), term_count,
        static_cast<const T*>(prefactors), static_cast<const T*>(prefactor_derivatives_center),
        static_cast<const T*>(prefactor_derivatives_neighbor), static_cast<const T*>(radial_directions),
        static_cast<const T*>(edge_weights), static_cast<const T*>(edge_weight_derivatives), edge_count, term_groups,
        term_channels, channel_count, static_cast<const T*>(edge_adjoint), static_cast<T*>(position_adjoint),
        static_cast<T*>(charge_center_adjoint), static_cast<T*>(charge_neighbor_adjoint), status);
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}
