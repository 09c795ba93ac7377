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

__device__ __forceinline__ void cmac(double2& acc, double c, double2 v) {
  acc.x = fma(c, v.x, acc.x);
  acc.y = fma(c, v.y, acc.y);
}

// acc += x * t (complex multiply-add)
__device__ __forceinline__ void cfma(double2& acc, double2 x, double2 t) {
  acc.x = fma(x.x, t.x, fma(-x.y, t.y, acc.x));
  acc.y = fma(x.x, t.y, fma(x.y, t.x, acc.y));
}

// Coefficient row of one prefix: NC doubles per j, padded to an even count so
// that a 16-byte load returns two coefficients (packing.py lays rows out so).
template <int DS, int NC>
struct RowWidth {
  static constexpr int value = NC == 2 ? 2 * DS : ((DS + 1) & ~1);
};

// Symmetric output of radial channel values x (x[i * stride] = component i
// of A[n, l]): sum_q coeff_q prod_i x_i^{k_qi}, the powers of each distinct
// input component multiplied in increasing component order
// (ye3t_runtime_core.cpp:5279).  Factors are 4 x u8 component indices
// (repeated for powers, 255 = unused).
__device__ __forceinline__ double2 sym_output(const y3b_ace_tables& t, int tb, int te, const double2* x,
                                              int stride) {
  double2 acc = make_double2(0.0, 0.0);
  for (int q = tb; q < te; ++q) {
    const uint32_t f = __ldg(t.sym_term_factors + q);
    double2 m = make_double2(__ldg(t.sym_term_coeff + q), 0.0);
    int k = 0;
    while (k < 4) {
      const int ci = (f >> (8 * k)) & 255;
      if (ci == 255) break;
      const double2 xv = x[ci * stride];
      double2 pw = xv;
      ++k;
      while (k < 4 && int((f >> (8 * k)) & 255) == ci) {
        pw = mul(pw, xv);
        ++k;
      }
      m = mul(m, pw);
    }
    acc = add(acc, m);
  }
  return acc;
}

}  // namespace y3b
