// Fused ACE evaluation: A-basis density (kernel 1) and multi-word factorized
// schedule bundle (kernel 2).
#include "edge_math.cuh"
#include "neighbors.cuh"

namespace y3b {

constexpr int kMaxNmax = 16;

// Warps per CTA of the density kernel, sized to keep its static shared memory
// under 48 KB.
template <int LMAX>
struct DensityWarps {
  static constexpr int value = LMAX >= 3 ? 2 : 4;
};

// ---------------------------------------------------------------------------
// Kernel 1: A-basis density.  One warp per centre atom.  Pass 1: lanes over
// up to 32 edges of the row compute p[z_j] R_n(r) and Yc_lm(r_hat) into
// warp-private shared memory.  Pass 2: lanes over the nmax*(lmax+1)^2 outputs
// accumulate those edges in CSR order.  A is written once per atom with
// coalesced stores; no atomics.
// ---------------------------------------------------------------------------
template <int LMAX>
__global__ void __launch_bounds__(32 * DensityWarps<LMAX>::value) ace_density_kernel(
    const double* __restrict__ pos, const int32_t* __restrict__ species, int64_t N,
    int64_t center_begin, int64_t count, double box, const int64_t* __restrict__ row_off,
    const int32_t* __restrict__ nbr, const double* __restrict__ pref, int64_t S, int nmax,
    double rc, double lam, ShNorm nrm, double2* __restrict__ A, int32_t* status) {
  constexpr int W = (LMAX + 1) * (LMAX + 1);
  constexpr int kOutPerLane = (kMaxNmax * W + 31) / 32;
  constexpr int kDensityWarps = DensityWarps<LMAX>::value;
  __shared__ double s_rad[kDensityWarps][32][kMaxNmax + 1];
  __shared__ double2 s_y[kDensityWarps][32][W];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int nout = nmax * W;
  const int64_t row0 = row_off[0];
  const int64_t warp = blockIdx.x * int64_t(kDensityWarps) + wib;
  const int64_t nwarps = int64_t(gridDim.x) * kDensityWarps;
  for (int64_t a = warp; a < count; a += nwarps) {
    const int64_t i = center_begin + a;
    const int64_t b = row_off[a] - row0, e = row_off[a + 1] - row0;
    double2 acc[kOutPerLane];
#pragma unroll
    for (int k = 0; k < kOutPerLane; ++k) acc[k] = make_double2(0.0, 0.0);
    for (int64_t c0 = b; c0 < e; c0 += 32) {
      const int nedge = (e - c0) < 32 ? int(e - c0) : 32;
      if (lane < nedge) {
        const int64_t j = nbr[c0 + lane];
        double rv[kMaxNmax + 1];
        double2 yc[W];
        double p = 0.0;
        if (j < 0 || j >= N) {
          if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
          for (int k = 0; k <= nmax; ++k) rv[k] = 0.0;
#pragma unroll
          for (int k = 0; k < W; ++k) yc[k] = make_double2(0.0, 0.0);
        } else {
          double d[3];
          min_image(pos, i, j, box, d);
          const double r = sqrt(dist2(d));
          const int zj = species[j];
          p = (zj >= 0 && zj < S) ? pref[zj] : 0.0;
          radial_basis<double>(r, rc, lam, nmax, rv, nullptr);
          const double sr = r > 1e-12 ? r : 1e-12;
          double v[W];
          real_sh_unit<double, LMAX>(d[0] / sr, d[1] / sr, d[2] / sr, nrm, v, nullptr);
          const double inv2 = 0.70710678118654752440084436210484903;
#pragma unroll
          for (int l = 0; l <= LMAX; ++l) {
            const int c = l * l + l;
            yc[c] = make_double2(v[c], 0.0);
#pragma unroll
            for (int m = 1; m <= l; ++m) {
              const double sg = (m & 1) ? -1.0 : 1.0;
              yc[c - m] = make_double2(inv2 * v[c + m], inv2 * v[c - m]);
              yc[c + m] = make_double2(sg * (inv2 * v[c + m]), sg * (inv2 * -v[c - m]));
            }
          }
        }
        for (int n = 0; n < nmax; ++n) s_rad[wib][lane][n] = p * rv[n + 1];
#pragma unroll
        for (int k = 0; k < W; ++k) s_y[wib][lane][k] = yc[k];
      }
      __syncwarp();
      for (int q = 0; q < nedge; ++q) {
#pragma unroll
        for (int k = 0; k < kOutPerLane; ++k) {
          const int o = lane + 32 * k;
          if (o < nout) {
            const int n = o / W, lm = o - n * W;
            const double rp = s_rad[wib][q][n];
            const double2 y = s_y[wib][q][lm];
            acc[k].x += rp * y.x;
            acc[k].y += rp * y.y;
          }
        }
      }
      __syncwarp();
    }
    double2* Ai = A + a * int64_t(nout);
#pragma unroll
    for (int k = 0; k < kOutPerLane; ++k) {
      const int o = lane + 32 * k;
      if (o < nout) Ai[o] = acc[k];
    }
  }
}

// ---------------------------------------------------------------------------
// Block pool: pool[idx][atom] (atom fastest) holding the A channels and every
// symmetric block of every radial channel.  One thread per atom.
// Symmetric terms multiply the coefficient by x_i^{k_i} for each distinct
// input component in increasing order, as ye3t_runtime_core.cpp:5279.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) ace_pool_kernel(y3b_ace_tables t, const double2* __restrict__ A,
                                                       int64_t N, double2* __restrict__ pool) {
  const int W = int((t.lmax + 1) * (t.lmax + 1));
  const int na = int(t.nmax) * W;
  for (int64_t a = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; a < N;
       a += int64_t(gridDim.x) * blockDim.x) {
    const double2* Aa = A + a * na;
    for (int idx = 0; idx < na; ++idx) pool[idx * N + a] = Aa[idx];
    for (int s = 0; s < t.sym_kind_count; ++s) {
      const int l = __ldg(t.sym_kind + 6 * s + 0);
      const int Lam = __ldg(t.sym_kind + 6 * s + 2);
      const int off = __ldg(t.sym_kind + 6 * s + 3);
      const int tb = __ldg(t.sym_kind + 6 * s + 4), te = __ldg(t.sym_kind + 6 * s + 5);
      const int dimo = 2 * Lam + 1;
      for (int n = 0; n < t.nmax; ++n) {
        const double2* x = Aa + n * W + l * l;
        for (int o = 0; o < dimo; ++o) pool[int64_t(off + n * dimo + o) * N + a] = make_double2(0.0, 0.0);
        for (int q = tb; q < te; ++q) {
          const int o = __ldg(t.sym_term_output + q);
          const uint32_t f = __ldg(t.sym_term_factors + q);
          const double c = __ldg(t.sym_term_coeff + q);
          double2 m = make_double2(c, 0.0);
          int k = 0;
          while (k < 4) {
            const int ci = (f >> (8 * k)) & 255;
            if (ci == 255) break;
            double2 r = x[ci];
            ++k;
            while (k < 4 && int((f >> (8 * k)) & 255) == ci) {
              r = mul(r, x[ci]);
              ++k;
            }
            m = mul(m, r);
          }
          double2* dst = pool + int64_t(off + n * dimo + o) * N + a;
          *dst = add(*dst, m);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Kernel 2: every word's schedule on blocks from the pool.  One thread per
// atom; the whole warp walks the same word/component/term sequence, so all
// table reads are uniform and every pool read is a coalesced 512-byte row
// segment.  MODE 0 writes features [N, F]; MODE 1 reduces to per-atom energy.
// ---------------------------------------------------------------------------
template <int MODE>
__global__ void __launch_bounds__(128) ace_eval_kernel(y3b_ace_tables t, const double2* __restrict__ pool,
                                                       int64_t N, double2* __restrict__ feats,
                                                       const int32_t* __restrict__ species,
                                                       const double* __restrict__ weights, int64_t S,
                                                       double* __restrict__ energy) {
  const int64_t a = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  const bool live = a < N;
  const int64_t aa = live ? a : 0;
  const double2* P = pool + aa;
  int z = 0;
  if (MODE == 1 && live) {
    z = species[aa];
    if (z < 0 || z >= S) z = 0;
  }
  double e_acc = 0.0;
  for (int64_t w = 0; w < t.word_count; ++w) {
    const int p = __ldg(t.word_pattern + w);
    const int B = __ldg(t.pattern_block_count + p);
    const int c0 = __ldg(t.pattern_comp_begin + p), c1 = __ldg(t.pattern_comp_begin + p + 1);
    const int lb = __ldg(t.word_label_base + w);
    const int64_t fo = __ldg(t.word_feature_offset + w);
    for (int c = c0; c < c1; ++c) {
      const int label = __ldg(t.comp_label + c);
      const int4 base = __ldg(reinterpret_cast<const int4*>(t.label_bases) + (lb + label));
      double2 acc = make_double2(0.0, 0.0);
      const int tb = __ldg(t.comp_term_begin + c), te = __ldg(t.comp_term_begin + c + 1);
      for (int q = tb; q < te; ++q) {
        const uint32_t mm = __ldg(t.term_m + q);
        const double cf = __ldg(t.term_coeff + q);
        double2 v = P[int64_t(base.x + int(mm & 255)) * N];
        v = make_double2(cf * v.x, cf * v.y);
        if (B > 1) v = mul(v, P[int64_t(base.y + int((mm >> 8) & 255)) * N]);
        if (B > 2) v = mul(v, P[int64_t(base.z + int((mm >> 16) & 255)) * N]);
        if (B > 3) v = mul(v, P[int64_t(base.w + int(mm >> 24)) * N]);
        acc = add(acc, v);
      }
      if (MODE == 0) {
        if (live) feats[aa * t.feature_count + fo + (c - c0)] = acc;
      } else {
        e_acc += __ldg(weights + int64_t(z) * t.feature_count + fo + (c - c0)) * acc.x;
      }
    }
  }
  if (MODE == 1 && live) energy[aa] = e_acc;
}

int check_tables(const y3b_ace_tables* t) {
  Y3B_CHECK_ARG(t != nullptr, "null tables");
  Y3B_CHECK_ARG(t->nmax >= 1 && t->nmax <= kMaxNmax, "nmax must be in [1, %d]", kMaxNmax);
  Y3B_CHECK_ARG(t->lmax >= 0 && t->lmax <= 6, "lmax must be in [0, 6]");
  Y3B_CHECK_ARG(t->max_blocks >= 1 && t->max_blocks <= 4, "bundles with more than 4 blocks per word are not supported");
  Y3B_CHECK_ARG(t->word_count >= 0 && t->feature_count >= 0 && t->pool_size >= 0, "negative table size");
  return Y3B_OK;
}

}  // namespace y3b

using namespace y3b;

extern "C" int y3b_ace_density(const double* positions, const int32_t* species, int64_t atom_count,
                               int64_t center_begin, int64_t center_count, double box,
                               const int64_t* row_offsets, const int32_t* neighbors,
                               const double* species_prefactor, int64_t species_count, int64_t nmax,
                               int64_t lmax, double cutoff, double lambda, void* A, int32_t* status,
                               void* stream) {
  Y3B_CHECK_ARG(nmax >= 1 && nmax <= kMaxNmax, "nmax must be in [1, %d]", kMaxNmax);
  Y3B_CHECK_ARG(center_begin >= 0 && center_count >= 0 && center_begin + center_count <= atom_count,
                "bad centre range");
  Y3B_CHECK_ARG(box > 0 && cutoff > 0, "box and cutoff must be positive");
  if (center_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(positions && species && row_offsets && species_prefactor && A, "null pointer argument");
  const ShNorm nrm = make_sh_norm();
  cudaStream_t s = as_stream(stream);
#define Y3B_DENSITY_CASE(L)                                                                     \
  case L:                                                                                       \
    ace_density_kernel<L><<<int(std::min<int64_t>((center_count + DensityWarps<L>::value - 1) / \
                                                      DensityWarps<L>::value,                   \
                                                  int64_t(kSMs) * 128)),                        \
                            32 * DensityWarps<L>::value, 0, s>>>(positions, species, atom_count, center_begin, \
                                                   center_count, box, row_offsets, neighbors,    \
                                                   species_prefactor, species_count, int(nmax),  \
                                                   cutoff, lambda, nrm,                          \
                                                   static_cast<double2*>(A), status);            \
    break;
  switch (lmax) {
    Y3B_DENSITY_CASE(0)
    Y3B_DENSITY_CASE(1)
    Y3B_DENSITY_CASE(2)
    Y3B_DENSITY_CASE(3)
    Y3B_DENSITY_CASE(4)
    default:
      return fail(Y3B_ERR_UNSUPPORTED, "ace_density: lmax %lld not built (0..4)", (long long)lmax);
  }
#undef Y3B_DENSITY_CASE
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_ace_pool(const y3b_ace_tables* tables, const void* A, int64_t atom_count, void* pool,
                            void* stream) {
  if (int rc = check_tables(tables)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && pool, "null pointer argument");
  ace_pool_kernel<<<grid_for(atom_count, 128), 128, 0, as_stream(stream)>>>(
      *tables, static_cast<const double2*>(A), atom_count, static_cast<double2*>(pool));
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_ace_features(const y3b_ace_tables* tables, const void* pool, int64_t atom_count,
                                void* features, void* stream) {
  if (int rc = check_tables(tables)) return rc;
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(pool && features, "null pointer argument");
  const int threads = 128;
  const int64_t grid = (atom_count + threads - 1) / threads;
  ace_eval_kernel<0><<<int(grid), threads, 0, as_stream(stream)>>>(
      *tables, static_cast<const double2*>(pool), atom_count, static_cast<double2*>(features),
      nullptr, nullptr, 0, nullptr);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_ace_energy(const y3b_ace_tables* tables, const void* pool, int64_t atom_count,
                              const int32_t* species, const double* weights, int64_t species_count,
                              double* energy, void* stream) {
  if (int rc = check_tables(tables)) return rc;
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(pool && species && weights && energy && species_count > 0, "null pointer argument");
  const int threads = 128;
  const int64_t grid = (atom_count + threads - 1) / threads;
  ace_eval_kernel<1><<<int(grid), threads, 0, as_stream(stream)>>>(
      *tables, static_cast<const double2*>(pool), atom_count, nullptr, species, weights, species_count,
      energy);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}
