// Evaluation items of the B-basis kernels (forward in ace.cu, adjoint in
// ace_grad.cu); the layout is written by ye3t_b200/packing.py.
#pragma once

#include "common.cuh"

namespace y3b {

struct Item {
  int sel, d0, d1, dl, K, coef, f0, f1;
  int b0, b1, b2, b3;
};

__device__ __forceinline__ Item load_item(const int4* __restrict__ items, int64_t i) {
  const int4 a = __ldg(items + 4 * i), b = __ldg(items + 4 * i + 1), c = __ldg(items + 4 * i + 2);
  Item it;
  it.sel = a.x; it.d0 = a.y; it.d1 = a.z; it.dl = a.w;
  it.K = b.x; it.coef = b.y; it.f0 = b.z; it.f1 = b.w;
  it.b0 = c.x; it.b1 = c.y; it.b2 = c.z; it.b3 = c.w;
  return it;
}

// Complex type of a real type, and its zero.
template <typename R> struct Cplx;
template <> struct Cplx<float> { using type = float2; };
template <> struct Cplx<double> { using type = double2; };
template <typename R> using Cx2 = typename Cplx<R>::type;
using CoefPair = double2;  // two fp64 coefficients read with one 16-byte load

template <typename C2> __device__ __forceinline__ C2 cz();
template <> __device__ __forceinline__ float2 cz<float2>() { return make_float2(0.f, 0.f); }
template <> __device__ __forceinline__ double2 cz<double2>() { return make_double2(0.0, 0.0); }

__device__ __forceinline__ void cmac(double2& acc, double c, double2 v) {
  acc.x = fma(c, v.x, acc.x);
  acc.y = fma(c, v.y, acc.y);
}
__device__ __forceinline__ void cmac(float2& acc, float c, float2 v) {
  acc.x = fmaf(c, v.x, acc.x);
  acc.y = fmaf(c, v.y, acc.y);
}

// acc += x * t (complex multiply-add)
__device__ __forceinline__ void cfma(double2& acc, double2 x, double2 t) {
  acc.x = fma(x.x, t.x, fma(-x.y, t.y, acc.x));
  acc.y = fma(x.x, t.y, fma(x.y, t.x, acc.y));
}
__device__ __forceinline__ void cfma(float2& acc, float2 x, float2 t) {
  acc.x = fmaf(x.x, t.x, fmaf(-x.y, t.y, acc.x));
  acc.y = fmaf(x.x, t.y, fmaf(x.y, t.x, acc.y));
}

// Coefficient row of one prefix: NC doubles per j, padded to an even count so
// that a 16-byte load returns two coefficients (packing.py lays rows out so).
template <int DS, int NC>
struct RowWidth {
  static constexpr int value = NC == 2 ? 2 * DS : ((DS + 1) & ~1);
};

// Symmetric output of radial channel values x (x[i * stride] = component i
// of A[n, l]): sum_q coeff_q prod_i x_i^{k_qi} (the grouped monomial tables
// of ye3t_runtime_core.cpp:5279).  Factors are 4 x u8 component indices
// (repeated for powers, 255 = unused), read with the coefficients from the
// given addresses (shared-memory copies of the tables).  Each monomial is its
// coefficient times its factors multiplied in order, with no data-dependent
// loop (threads of one warp may follow different factor patterns), two terms
// per iteration into separate sums.
template <typename C2>
__device__ __forceinline__ C2 sym_output_tab(const uint32_t* fac, const double* co, int tb, int te, const C2* x,
                                             int stride) {
  using R = decltype(C2{}.x);
  C2 acc[2] = {cz<C2>(), cz<C2>()};
#pragma unroll 1
  for (int q0 = tb; q0 < te; q0 += 2) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int q = q0 + h < te ? q0 + h : q0;  // a lone last term runs twice, the copy with weight 0
      const uint32_t f = fac[q];
      C2 m = cz<C2>();
      m.x = q0 + h < te ? R(co[q]) : R(0);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int ci = (f >> (8 * k)) & 255;
        if (ci != 255) m = mul(m, x[ci * stride]);
      }
      acc[h] = add(acc[h], m);
    }
  }
  return add(acc[0], acc[1]);
}

}  // namespace y3b
