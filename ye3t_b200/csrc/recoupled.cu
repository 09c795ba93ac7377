// Recoupled B-basis adjoint: per-atom energies and G = dE/dA of a scalar ACE
// bundle whose features are written as contractions of coupled channel pairs,
// F_f = sum_L W[f, L] sum_M (-1)^M I_A^L[M] I_B^L[-M] (the plan and its tables
// are built on the host by ye3t_b200/recoupling.py).  The energy of atom i is
// e_i = Re(Q_i), Q = sum_d k[z_i, d] T_d with real weights k folded from the
// readout.  Q is quadratic in the coupled components I, so with
// gI = dQ/dI, Q = (1/2) sum_c I_c gI_c, and one sweep gives both.
//
// One CTA per atom (grid-stride), one pass per intermediate L:
//   1. the pass's components I (pairs coupled through their Clebsch-Gordan
//      terms, single channels copied, the unit) into shared memory;
//   2. every component's adjoint gI[c] = (-1)^M sum over its segment's
//      contraction list of k[d] I[partner][-M]: each component owns its sum,
//      so no atomics and a fixed summation order; the energy share
//      Re(I[c] gI[c]) accumulates per thread;
//   3. each A-row entry adds its Clebsch-Gordan back-propagation terms
//      (owner-computes again).
// Every table index the kernel follows is checked against the pass or the
// array it addresses; an entry outside them sets Y3B_STATUS_TABLE and is
// skipped, so a damaged table cannot reach outside shared memory.
#include <algorithm>

#include "common.cuh"

namespace y3b {
namespace {

constexpr int kRecThreads = 256;

struct RecTabs {
  int32_t pass_count, max_pass_components, row_width, dot_count;
  int64_t component_count, cg_count, own_count, bp_count;
  const int32_t* pass_begin;
  const int4* comp;  // two int4 per component: (a, b, cg_begin, cg_count), (m, own_begin, own_count, 0)
  const int32_t* cg_index;
  const double* cg_value;
  const int2* own;  // (partner's first local component, contraction)
  const int32_t* bp_begin;
  const int32_t* bp_gi;
  const int32_t* bp_other;
  const double* bp_value;
  int64_t feature_count, feat_count;
  const int32_t* dot_begin;
  const int4* dot;  // (A's first local component, B's, feature range begin, count)
  const int32_t* feat_index;
  const double* feat_weight;
};

// Fixed-order block sum of one double per thread (warp shuffles, then the
// warps in order); the result is valid in thread 0.
__device__ __forceinline__ double block_sum(double v, double* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  double s = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < kRecThreads / 32; ++w) s += red[w];
  return s;
}

// Shared-memory arrays hold NA atoms side by side: entry e of atom a at
// [e * NA + a].  A CTA takes atoms [g NA, g NA + NA); every table entry it
// loads (coupling term, contraction-list entry, back-propagation entry,
// contraction) serves all NA atoms, and the NA sums are independent chains.
template <int NA>
__device__ __forceinline__ void build_components(const RecTabs& t, const double2* sA, double2* sI, int c0, int nc,
                                                 int W, bool& bad) {
  for (int c = threadIdx.x; c < nc; c += kRecThreads) {
    const int4 d = __ldg(t.comp + 2 * (c0 + c));
    double2 v[NA];
#pragma unroll
    for (int a = 0; a < NA; ++a) v[a] = make_double2(d.x < 0 ? 1.0 : 0.0, 0.0);
    if (d.x < 0) {
    } else if (d.w == 0) {
      if (d.x < W) {
#pragma unroll
        for (int a = 0; a < NA; ++a) v[a] = sA[d.x * NA + a];
      } else {
        bad = true;
      }
    } else if (d.z < 0 || int64_t(d.z) + d.w > t.cg_count || d.y < 0) {
      bad = true;
    } else {
      for (int q = d.z; q < d.z + d.w; ++q) {
        const int ix = __ldg(t.cg_index + q);
        const int ia = d.x + (ix & 255), ib = d.y + (ix >> 8);
        if (ia >= W || ib < 0 || ib >= W) {
          bad = true;
          continue;
        }
        const double cv = __ldg(t.cg_value + q);
#pragma unroll
        for (int a = 0; a < NA; ++a) {
          const double2 p = mul(sA[ia * NA + a], sA[ib * NA + a]);
          v[a].x = fma(cv, p.x, v[a].x);
          v[a].y = fma(cv, p.y, v[a].y);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < NA; ++a) sI[c * NA + a] = v[a];
  }
}

// The CTA's atoms: count of valid ones, their weight rows (species outside
// the range set the status and use species 0), and their A rows in sA.
template <int NA>
__device__ __forceinline__ int load_atoms(int64_t first, int64_t atom_count, int W, const double2* A,
                                          const int32_t* species, const double* k, int64_t species_count,
                                          int32_t dot_count, double2* sA, double2* sGA, const double** kz,
                                          int32_t* status) {
  const int nv = int(atom_count - first < NA ? atom_count - first : NA);
#pragma unroll
  for (int a = 0; a < NA; ++a) {
    int z = 0;
    if (species != nullptr && a < nv) {
      z = species[first + a];
      if (z < 0 || z >= species_count) {
        if (threadIdx.x == 0 && status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
        z = 0;
      }
    }
    kz[a] = k == nullptr ? nullptr : k + int64_t(z) * dot_count;
  }
  for (int i = threadIdx.x; i < W * NA; i += kRecThreads) {
    const int a = i % NA, e = i / NA;
    sA[i] = a < nv ? A[(first + a) * W + e] : make_double2(0.0, 0.0);
    if (sGA != nullptr) sGA[i] = make_double2(0.0, 0.0);
  }
  return nv;
}

template <int NA>
__global__ void __launch_bounds__(kRecThreads)
recoupled_energy_grad_kernel(RecTabs t, const double2* __restrict__ A, int64_t atom_count,
                             const int32_t* __restrict__ species, const double* __restrict__ k,
                             int64_t species_count, double* __restrict__ energy, double2* __restrict__ G,
                             int32_t* status) {
  extern __shared__ double2 rec_smem[];
  __shared__ double red[kRecThreads / 32];
  const int W = t.row_width;
  const int maxc = t.max_pass_components;
  double2* sA = rec_smem;          // [W][NA] the atoms' A rows
  double2* sGA = sA + W * NA;      // [W][NA] dE/dA of the rows
  double2* sI = sGA + W * NA;      // [maxc][NA] components of the pass
  double2* sG = sI + maxc * NA;    // [maxc][NA] their adjoints
  const int tid = threadIdx.x;
  const int64_t groups = (atom_count + NA - 1) / NA;
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t first = grp * NA;
    const double* kz[NA];
    const int nv = load_atoms<NA>(first, atom_count, W, A, species, k, species_count, t.dot_count, sA, sGA, kz,
                                  status);
    double ep[NA];
#pragma unroll
    for (int a = 0; a < NA; ++a) ep[a] = 0.0;
    bool bad = false;
    __syncthreads();
    for (int L = 0; L < t.pass_count; ++L) {
      const int c0 = t.pass_begin[L];
      const int nc = t.pass_begin[L + 1] - c0;
      if (c0 < 0 || nc < 0 || nc > maxc || int64_t(c0) + nc > t.component_count) {
        bad = true;  // uniform over the block: every thread reads the same entries
        continue;
      }
      // 1. components
      build_components<NA>(t, sA, sI, c0, nc, W, bad);
      __syncthreads();
      // 2. adjoints of the components and the energy shares
      for (int c = tid; c < nc; c += kRecThreads) {
        const int4 d = __ldg(t.comp + 2 * (c0 + c) + 1);
        double2 acc[NA];
#pragma unroll
        for (int a = 0; a < NA; ++a) acc[a] = make_double2(0.0, 0.0);
        if (d.y < 0 || d.z < 0 || int64_t(d.y) + d.z > t.own_count) {
          bad = true;
        } else {
          const int r = 2 * L - d.x;
          for (int q = d.y; q < d.y + d.z; ++q) {
            const int2 e = __ldg(t.own + q);
            const int p = e.x + r;
            if (p < 0 || p >= nc || e.y < 0 || e.y >= t.dot_count) {
              bad = true;
              continue;
            }
#pragma unroll
            for (int a = 0; a < NA; ++a) {
              const double kk = __ldg(kz[a] + e.y);
              const double2 v = sI[p * NA + a];
              acc[a].x = fma(kk, v.x, acc[a].x);
              acc[a].y = fma(kk, v.y, acc[a].y);
            }
          }
        }
        const double sgn = ((d.x - L) & 1) ? -1.0 : 1.0;
#pragma unroll
        for (int a = 0; a < NA; ++a) {
          acc[a].x *= sgn;
          acc[a].y *= sgn;
          sG[c * NA + a] = acc[a];
          const double2 iv = sI[c * NA + a];
          ep[a] = fma(iv.x, acc[a].x, ep[a]);
          ep[a] = fma(-iv.y, acc[a].y, ep[a]);
        }
      }
      __syncthreads();
      // 3. back-propagation into the A rows (each entry owns its sum)
      for (int i = tid; i < W; i += kRecThreads) {
        const int64_t at = int64_t(L) * W + i;
        const int b0 = t.bp_begin[at], b1 = t.bp_begin[at + 1];
        if (b0 < 0 || b1 < b0 || int64_t(b1) > t.bp_count) {
          bad = true;
          continue;
        }
        double2 ga[NA];
#pragma unroll
        for (int a = 0; a < NA; ++a) ga[a] = sGA[i * NA + a];
        for (int q = b0; q < b1; ++q) {
          const int gi = __ldg(t.bp_gi + q);
          const int o = __ldg(t.bp_other + q);
          if (gi < 0 || gi >= nc || o >= W) {
            bad = true;
            continue;
          }
          const double cv = __ldg(t.bp_value + q);
#pragma unroll
          for (int a = 0; a < NA; ++a) {
            const double2 g = sG[gi * NA + a];
            const double2 term = o < 0 ? g : mul(g, sA[o * NA + a]);
            ga[a].x = fma(cv, term.x, ga[a].x);
            ga[a].y = fma(cv, term.y, ga[a].y);
          }
        }
#pragma unroll
        for (int a = 0; a < NA; ++a) sGA[i * NA + a] = ga[a];
      }
      __syncthreads();
    }
    if (bad && status) atomicOr(status, Y3B_STATUS_TABLE);
    for (int i = tid; i < W * NA; i += kRecThreads) {
      const int a = i % NA, e = i / NA;
      if (a < nv) G[(first + a) * W + e] = sGA[i];
    }
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      const double total = block_sum(ep[a], red);
      if (tid == 0 && a < nv) energy[first + a] = 0.5 * total;
      __syncthreads();
    }
  }
}

// Forward pass: per L the components, then every contraction of the pass once,
// T_d = sum_M (-1)^M I_A[M] I_B[-M]; the energies e = Re(sum_d k[z, d] T_d)
// (kFeatures false) or the features F[f] += W[f, d] T_d (kFeatures true: a word
// has at most one contraction per L and a feature belongs to one word, so each
// feature has one writer per pass and the passes are ordered by barriers).
template <bool kFeatures, int NA>
__global__ void __launch_bounds__(kRecThreads)
recoupled_forward_kernel(RecTabs t, const double2* __restrict__ A, int64_t atom_count,
                         const int32_t* __restrict__ species, const double* __restrict__ k, int64_t species_count,
                         double* __restrict__ energy, double2* __restrict__ features, int32_t* status) {
  extern __shared__ double2 rec_smem[];
  __shared__ double red[kRecThreads / 32];
  const int W = t.row_width;
  double2* sA = rec_smem;     // [W][NA]
  double2* sI = sA + W * NA;  // [max_pass_components][NA]
  const int tid = threadIdx.x;
  const int64_t groups = (atom_count + NA - 1) / NA;
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t first = grp * NA;
    const double* kz[NA];
    const int nv = load_atoms<NA>(first, atom_count, W, A, kFeatures ? nullptr : species, kFeatures ? nullptr : k,
                                  species_count, t.dot_count, sA, nullptr, kz, status);
    if constexpr (kFeatures) {
      for (int64_t i = tid; i < int64_t(nv) * t.feature_count; i += kRecThreads)
        features[first * t.feature_count + i] = make_double2(0.0, 0.0);
    }
    double ep[NA];
#pragma unroll
    for (int a = 0; a < NA; ++a) ep[a] = 0.0;
    bool bad = false;
    __syncthreads();
    for (int L = 0; L < t.pass_count; ++L) {
      const int c0 = t.pass_begin[L];
      const int nc = t.pass_begin[L + 1] - c0;
      const int d0 = t.dot_begin[L];
      const int nd = t.dot_begin[L + 1] - d0;
      if (c0 < 0 || nc < 0 || nc > t.max_pass_components || int64_t(c0) + nc > t.component_count || d0 < 0 ||
          nd < 0 || int64_t(d0) + nd > t.dot_count) {
        bad = true;  // uniform over the block
        continue;
      }
      build_components<NA>(t, sA, sI, c0, nc, W, bad);
      __syncthreads();
      for (int j = tid; j < nd; j += kRecThreads) {
        const int4 q = __ldg(t.dot + d0 + j);
        if (q.x < 0 || q.y < 0 || q.x + 2 * L >= nc || q.y + 2 * L >= nc) {
          bad = true;
          continue;
        }
        double2 T[NA];
#pragma unroll
        for (int a = 0; a < NA; ++a) T[a] = make_double2(0.0, 0.0);
        for (int m = 0; m <= 2 * L; ++m) {  // m = M + L
          const double sgn = ((m - L) & 1) ? -1.0 : 1.0;
#pragma unroll
          for (int a = 0; a < NA; ++a) {
            const double2 p = mul(sI[(q.x + m) * NA + a], sI[(q.y + 2 * L - m) * NA + a]);
            T[a].x = fma(sgn, p.x, T[a].x);
            T[a].y = fma(sgn, p.y, T[a].y);
          }
        }
        if constexpr (kFeatures) {
          if (q.z < 0 || q.w < 0 || int64_t(q.z) + q.w > t.feat_count) {
            bad = true;
            continue;
          }
          for (int z = q.z; z < q.z + q.w; ++z) {
            const int f = __ldg(t.feat_index + z);
            if (f < 0 || f >= t.feature_count) {
              bad = true;
              continue;
            }
            const double wv = __ldg(t.feat_weight + z);
#pragma unroll
            for (int a = 0; a < NA; ++a) {
              if (a < nv) {
                double2* slot = features + (first + a) * t.feature_count + f;
                double2 v = *slot;
                v.x = fma(wv, T[a].x, v.x);
                v.y = fma(wv, T[a].y, v.y);
                *slot = v;
              }
            }
          }
        } else {
#pragma unroll
          for (int a = 0; a < NA; ++a) ep[a] = fma(__ldg(kz[a] + d0 + j), T[a].x, ep[a]);
        }
      }
      __syncthreads();
    }
    if (bad && status) atomicOr(status, Y3B_STATUS_TABLE);
    if constexpr (!kFeatures) {
#pragma unroll
      for (int a = 0; a < NA; ++a) {
        const double total = block_sum(ep[a], red);
        if (tid == 0 && a < nv) energy[first + a] = total;
        __syncthreads();
      }
    } else {
      __syncthreads();
    }
  }
}

}  // namespace
}  // namespace y3b

using namespace y3b;

namespace {

int check_tables(const y3b_recoupled_tables* tables) {
  Y3B_CHECK_ARG(tables != nullptr, "null tables");
  const y3b_recoupled_tables& t = *tables;
  Y3B_CHECK_ARG(t.pass_count >= 1 && t.pass_count <= 64, "pass_count must be in [1, 64]");
  Y3B_CHECK_ARG(t.row_width >= 1 && t.row_width <= 4096, "row_width must be in [1, 4096]");
  Y3B_CHECK_ARG(t.max_pass_components >= 1 && t.dot_count >= 1 && t.feature_count >= 1, "empty recoupled tables");
  Y3B_CHECK_ARG(t.component_count >= 1 && t.cg_count >= 0 && t.own_count >= 0 && t.bp_count >= 0 &&
                    t.feat_count >= 0,
                "negative table sizes");
  Y3B_CHECK_ARG(t.pass_begin && t.comp && t.own && t.bp_begin && t.bp_gi && t.bp_other && t.bp_value &&
                    t.dot_begin && t.dot && (t.cg_count == 0 || (t.cg_index && t.cg_value)) &&
                    (t.feat_count == 0 || (t.feat_index && t.feat_weight)),
                "null table pointer");
  Y3B_CHECK_ARG(reinterpret_cast<uintptr_t>(t.comp) % 16 == 0 && reinterpret_cast<uintptr_t>(t.dot) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(t.own) % 8 == 0,
                "comp and dot must be 16-byte and own 8-byte aligned");
  return Y3B_OK;
}

RecTabs device_view(const y3b_recoupled_tables& t) {
  return RecTabs{t.pass_count, t.max_pass_components, t.row_width, t.dot_count,
                 t.component_count, t.cg_count, t.own_count, t.bp_count,
                 t.pass_begin, reinterpret_cast<const int4*>(t.comp), t.cg_index, t.cg_value,
                 reinterpret_cast<const int2*>(t.own), t.bp_begin, t.bp_gi, t.bp_other, t.bp_value,
                 t.feature_count, t.feat_count, t.dot_begin, reinterpret_cast<const int4*>(t.dot), t.feat_index,
                 t.feat_weight};
}

// Atoms per CTA: the tables' atoms_per_cta (0 means 1), in [1, 4].
int atoms_per_cta(const y3b_recoupled_tables& t, int& na) {
  na = t.atoms_per_cta == 0 ? 1 : t.atoms_per_cta;
  Y3B_CHECK_ARG(na >= 1 && na <= 4, "atoms_per_cta must be 0 (one) or in [1, 4]");
  return Y3B_OK;
}

template <typename Kernel>
int launch_grouped(Kernel kernel, size_t smem_per_atom, int na, int64_t atom_count, cudaStream_t s,
                   const RecTabs& rt, const void* A, const int32_t* species, const double* weights,
                   int64_t species_count, double* energy, void* out, int32_t* status) {
  const size_t smem = smem_per_atom * size_t(na);
  Y3B_CHECK_ARG(smem <= 224 * 1024,
                "recoupled pass needs %lld bytes of shared memory for %d atoms per CTA (max 224 KB)",
                (long long)smem, na);
  const int64_t groups = (atom_count + na - 1) / na;
  const int64_t grid = std::min<int64_t>(groups, int64_t(kSMs) * 64);
  Y3B_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  kernel<<<int(grid), kRecThreads, smem, s>>>(rt, static_cast<const double2*>(A), atom_count, species, weights,
                                              species_count, energy, static_cast<double2*>(out), status);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

template <bool kFeatures>
int launch_forward(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count, const int32_t* species,
                   const double* weights, int64_t species_count, double* energy, void* features, int32_t* status,
                   void* stream) {
  if (int rc = check_tables(tables)) return rc;
  const y3b_recoupled_tables& t = *tables;
  int na = 1;
  if (int rc = atoms_per_cta(t, na)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A != nullptr, "null A");
  if (kFeatures) {
    Y3B_CHECK_ARG(features != nullptr, "null features");
  } else {
    Y3B_CHECK_ARG(species && weights && energy && species_count > 0, "null pointer argument");
  }
  const size_t per_atom = size_t(int64_t(t.row_width) + int64_t(t.max_pass_components)) * sizeof(double2);
  const RecTabs rt = device_view(t);
  cudaStream_t s = as_stream(stream);
  switch (na) {
    case 1: return launch_grouped(recoupled_forward_kernel<kFeatures, 1>, per_atom, 1, atom_count, s, rt, A,
                                  species, weights, species_count, energy, features, status);
    case 2: return launch_grouped(recoupled_forward_kernel<kFeatures, 2>, per_atom, 2, atom_count, s, rt, A,
                                  species, weights, species_count, energy, features, status);
    case 3: return launch_grouped(recoupled_forward_kernel<kFeatures, 3>, per_atom, 3, atom_count, s, rt, A,
                                  species, weights, species_count, energy, features, status);
    default: return launch_grouped(recoupled_forward_kernel<kFeatures, 4>, per_atom, 4, atom_count, s, rt, A,
                                   species, weights, species_count, energy, features, status);
  }
}

}  // namespace

extern "C" int y3b_ace_recoupled_energy(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count,
                                        const int32_t* species, const double* contraction_weights,
                                        int64_t species_count, double* energy, int32_t* status, void* stream) {
  return launch_forward<false>(tables, A, atom_count, species, contraction_weights, species_count, energy, nullptr,
                               status, stream);
}

extern "C" int y3b_ace_recoupled_features(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count,
                                          void* features, int32_t* status, void* stream) {
  return launch_forward<true>(tables, A, atom_count, nullptr, nullptr, 0, nullptr, features, status, stream);
}

extern "C" int y3b_ace_recoupled_energy_grad(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count,
                                             const int32_t* species, const double* contraction_weights,
                                             int64_t species_count, double* energy, void* dEdA, int32_t* status,
                                             void* stream) {
  if (int rc = check_tables(tables)) return rc;
  const y3b_recoupled_tables& t = *tables;
  int na = 1;
  if (int rc = atoms_per_cta(t, na)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && species && contraction_weights && energy && dEdA && species_count > 0,
                "null pointer argument");
  const size_t per_atom = size_t(2 * int64_t(t.row_width) + 2 * int64_t(t.max_pass_components)) * sizeof(double2);
  const RecTabs rt = device_view(t);
  cudaStream_t s = as_stream(stream);
  switch (na) {
    case 1: return launch_grouped(recoupled_energy_grad_kernel<1>, per_atom, 1, atom_count, s, rt, A, species,
                                  contraction_weights, species_count, energy, dEdA, status);
    case 2: return launch_grouped(recoupled_energy_grad_kernel<2>, per_atom, 2, atom_count, s, rt, A, species,
                                  contraction_weights, species_count, energy, dEdA, status);
    case 3: return launch_grouped(recoupled_energy_grad_kernel<3>, per_atom, 3, atom_count, s, rt, A, species,
                                  contraction_weights, species_count, energy, dEdA, status);
    default: return launch_grouped(recoupled_energy_grad_kernel<4>, per_atom, 4, atom_count, s, rt, A, species,
                                   contraction_weights, species_count, energy, dEdA, status);
  }
}
