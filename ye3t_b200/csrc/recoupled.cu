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
#include "recoupled_kernels.cuh"


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
