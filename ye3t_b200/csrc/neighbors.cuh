// Minimum-image displacement shared by the neighbour builder and the A-basis
// kernel.  Written with non-contracting intrinsics so that it rounds exactly
// like the serial CPU expression  x -= box * nearbyint(x / box)  and
// r2 = (d0*d0 + d1*d1) + d2*d2.
#pragma once

namespace y3b {

__device__ __forceinline__ void min_image(const double* __restrict__ pos, int64_t i, int64_t j,
                                          double box, double d[3]) {
#pragma unroll
  for (int a = 0; a < 3; ++a) {
    const double x = __dsub_rn(pos[3 * j + a], pos[3 * i + a]);
    d[a] = __dsub_rn(x, __dmul_rn(box, rint(__ddiv_rn(x, box))));
  }
}

__device__ __forceinline__ double dist2(const double d[3]) {
  return __dadd_rn(__dadd_rn(__dmul_rn(d[0], d[0]), __dmul_rn(d[1], d[1])), __dmul_rn(d[2], d[2]));
}

int cells_per_side(double box, double cutoff);

}  // namespace y3b
