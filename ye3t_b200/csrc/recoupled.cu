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
};

__global__ void __launch_bounds__(kRecThreads)
recoupled_energy_grad_kernel(RecTabs t, const double2* __restrict__ A, int64_t atom_count,
                             const int32_t* __restrict__ species, const double* __restrict__ k,
                             int64_t species_count, double* __restrict__ energy, double2* __restrict__ G,
                             int32_t* status) {
  extern __shared__ double2 rec_smem[];
  __shared__ double red[kRecThreads / 32];
  const int W = t.row_width;
  const int maxc = t.max_pass_components;
  double2* sA = rec_smem;      // [W] the atom's A row
  double2* sGA = sA + W;       // [W] dE/dA of the row
  double2* sI = sGA + W;       // [maxc] components of the pass
  double2* sG = sI + maxc;     // [maxc] their adjoints
  const int tid = threadIdx.x;
  for (int64_t atom = blockIdx.x; atom < atom_count; atom += gridDim.x) {
    int z = species[atom];
    if (z < 0 || z >= species_count) {
      if (tid == 0 && status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
      z = 0;
    }
    const double* kz = k + int64_t(z) * t.dot_count;
    const double2* Arow = A + atom * W;
    for (int i = tid; i < W; i += kRecThreads) {
      sA[i] = Arow[i];
      sGA[i] = make_double2(0.0, 0.0);
    }
    double ep = 0.0;
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
      for (int c = tid; c < nc; c += kRecThreads) {
        const int4 d = __ldg(t.comp + 2 * (c0 + c));
        double2 v = make_double2(0.0, 0.0);
        if (d.x < 0) {
          v.x = 1.0;
        } else if (d.w == 0) {
          if (d.x < W) v = sA[d.x];
          else bad = true;
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
            const double2 p = mul(sA[ia], sA[ib]);
            v.x = fma(cv, p.x, v.x);
            v.y = fma(cv, p.y, v.y);
          }
        }
        sI[c] = v;
      }
      __syncthreads();
      // 2. adjoints of the components and the energy share
      for (int c = tid; c < nc; c += kRecThreads) {
        const int4 d = __ldg(t.comp + 2 * (c0 + c) + 1);
        double2 acc = make_double2(0.0, 0.0);
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
            const double kk = __ldg(kz + e.y);
            const double2 v = sI[p];
            acc.x = fma(kk, v.x, acc.x);
            acc.y = fma(kk, v.y, acc.y);
          }
        }
        if ((d.x - L) & 1) {
          acc.x = -acc.x;
          acc.y = -acc.y;
        }
        sG[c] = acc;
        const double2 iv = sI[c];
        ep = fma(iv.x, acc.x, ep);
        ep = fma(-iv.y, acc.y, ep);
      }
      __syncthreads();
      // 3. back-propagation into the A row (each entry owns its sum)
      for (int i = tid; i < W; i += kRecThreads) {
        const int64_t at = int64_t(L) * W + i;
        const int b0 = t.bp_begin[at], b1 = t.bp_begin[at + 1];
        if (b0 < 0 || b1 < b0 || int64_t(b1) > t.bp_count) {
          bad = true;
          continue;
        }
        double2 ga = sGA[i];
        for (int q = b0; q < b1; ++q) {
          const int gi = __ldg(t.bp_gi + q);
          const int o = __ldg(t.bp_other + q);
          if (gi < 0 || gi >= nc || o >= W) {
            bad = true;
            continue;
          }
          const double cv = __ldg(t.bp_value + q);
          const double2 g = sG[gi];
          const double2 term = o < 0 ? g : mul(g, sA[o]);
          ga.x = fma(cv, term.x, ga.x);
          ga.y = fma(cv, term.y, ga.y);
        }
        sGA[i] = ga;
      }
      __syncthreads();
    }
    if (bad && status) atomicOr(status, Y3B_STATUS_TABLE);
    for (int i = tid; i < W; i += kRecThreads) G[atom * W + i] = sGA[i];
    // energy: warp sums, then the warps in order (fixed order)
    for (int o = 16; o > 0; o >>= 1) ep += __shfl_xor_sync(0xffffffffu, ep, o);
    if ((tid & 31) == 0) red[tid >> 5] = ep;
    __syncthreads();
    if (tid == 0) {
      double s = 0.0;
      for (int w = 0; w < kRecThreads / 32; ++w) s += red[w];
      energy[atom] = 0.5 * s;
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace y3b

using namespace y3b;

extern "C" int y3b_ace_recoupled_energy_grad(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count,
                                             const int32_t* species, const double* contraction_weights,
                                             int64_t species_count, double* energy, void* dEdA, int32_t* status,
                                             void* stream) {
  Y3B_CHECK_ARG(tables != nullptr, "null tables");
  const y3b_recoupled_tables& t = *tables;
  Y3B_CHECK_ARG(t.pass_count >= 1 && t.pass_count <= 64, "pass_count must be in [1, 64]");
  Y3B_CHECK_ARG(t.row_width >= 1 && t.row_width <= 4096, "row_width must be in [1, 4096]");
  Y3B_CHECK_ARG(t.max_pass_components >= 1 && t.dot_count >= 1, "empty recoupled tables");
  Y3B_CHECK_ARG(t.component_count >= 1 && t.cg_count >= 0 && t.own_count >= 0 && t.bp_count >= 0,
                "negative table sizes");
  Y3B_CHECK_ARG(t.pass_begin && t.comp && t.own && t.bp_begin && t.bp_gi && t.bp_other && t.bp_value &&
                    (t.cg_count == 0 || (t.cg_index && t.cg_value)),
                "null table pointer");
  Y3B_CHECK_ARG(reinterpret_cast<uintptr_t>(t.comp) % 16 == 0 && reinterpret_cast<uintptr_t>(t.own) % 8 == 0,
                "comp must be 16-byte and own 8-byte aligned");
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && species && contraction_weights && energy && dEdA && species_count > 0,
                "null pointer argument");
  const size_t smem = size_t(2 * int64_t(t.row_width) + 2 * int64_t(t.max_pass_components)) * sizeof(double2);
  Y3B_CHECK_ARG(smem <= 224 * 1024, "recoupled pass needs %lld bytes of shared memory (max 224 KB)",
                (long long)smem);
  RecTabs rt{t.pass_count, t.max_pass_components, t.row_width, t.dot_count,
             t.component_count, t.cg_count, t.own_count, t.bp_count,
             t.pass_begin, reinterpret_cast<const int4*>(t.comp), t.cg_index, t.cg_value,
             reinterpret_cast<const int2*>(t.own), t.bp_begin, t.bp_gi, t.bp_other, t.bp_value};
  const int64_t grid = std::min<int64_t>(atom_count, int64_t(kSMs) * 64);
  cudaStream_t s = as_stream(stream);
  Y3B_CUDA_TRY(cudaFuncSetAttribute(recoupled_energy_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)));
  recoupled_energy_grad_kernel<<<int(grid), kRecThreads, smem, s>>>(
      rt, static_cast<const double2*>(A), atom_count, species, contraction_weights, species_count, energy,
      static_cast<double2*>(dEdA), status);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}
