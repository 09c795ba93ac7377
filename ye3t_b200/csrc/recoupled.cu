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
//      (owner-computes again; a long list is split over the threads that
//      step 3 would leave idle, and the parts are added in a fixed order).
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


// Launch shape from the tables: atoms per CTA (0 means 1; 1..4) and threads
// per CTA (0 means 256; 256 or 512).
template <typename T>
int launch_shape(const T& t, int& na, int& th) {
  na = t.atoms_per_cta == 0 ? 1 : t.atoms_per_cta;
  th = t.threads_per_cta == 0 ? 256 : t.threads_per_cta;
  Y3B_CHECK_ARG(na >= 1 && na <= 4, "atoms_per_cta must be 0 (one) or in [1, 4]");
  Y3B_CHECK_ARG(th == 256 || th == 512, "threads_per_cta must be 0 (256), 256 or 512");
  return Y3B_OK;
}

// Dynamic shared memory per atom of the adjoint passes: the A row and its
// adjoint, and two component regions that also hold step 3's W parts.
size_t grad_smem_per_atom(int64_t row_width, int64_t max_pass_components) {
  const int64_t cw = std::max(row_width, max_pass_components);
  return size_t(2 * row_width + 2 * cw) * sizeof(double2);
}

template <typename Kernel, typename Tabs>
int launch_grouped(Kernel kernel, int threads, size_t smem_per_atom, int na, int64_t atom_count, cudaStream_t s,
                   const Tabs& rt, const void* A, const int32_t* species, const double* weights,
                   int64_t species_count, double* energy, void* out, int32_t* status) {
  const size_t smem = smem_per_atom * size_t(na);
  Y3B_CHECK_ARG(smem <= 224 * 1024,
                "recoupled pass needs %lld bytes of shared memory for %d atoms per CTA (max 224 KB)",
                (long long)smem, na);
  const int64_t groups = (atom_count + na - 1) / na;
  const int64_t grid = std::min<int64_t>(groups, int64_t(kSMs) * 64);
  Y3B_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  kernel<<<int(grid), threads, smem, s>>>(rt, static_cast<const double2*>(A), atom_count, species, weights,
                                          species_count, energy, static_cast<double2*>(out), status);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

// One case per (atoms per CTA, threads per CTA) instance of a kernel template.
#define Y3B_REC_DISPATCH(KERNEL, ...)                                                                   \
  switch (na * 1000 + th) {                                                                             \
    case 1256: return launch_grouped(KERNEL(1, 256), 256, __VA_ARGS__);                                 \
    case 2256: return launch_grouped(KERNEL(2, 256), 256, __VA_ARGS__);                                 \
    case 3256: return launch_grouped(KERNEL(3, 256), 256, __VA_ARGS__);                                 \
    case 4256: return launch_grouped(KERNEL(4, 256), 256, __VA_ARGS__);                                 \
    case 1512: return launch_grouped(KERNEL(1, 512), 512, __VA_ARGS__);                                 \
    case 2512: return launch_grouped(KERNEL(2, 512), 512, __VA_ARGS__);                                 \
    case 3512: return launch_grouped(KERNEL(3, 512), 512, __VA_ARGS__);                                 \
    default: return launch_grouped(KERNEL(4, 512), 512, __VA_ARGS__);                                   \
  }

template <bool kFeatures>
int launch_forward(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count, const int32_t* species,
                   const double* weights, int64_t species_count, double* energy, void* features, int32_t* status,
                   void* stream) {
  if (int rc = check_tables(tables)) return rc;
  const y3b_recoupled_tables& t = *tables;
  int na = 1, th = 256;
  if (int rc = launch_shape(t, na, th)) return rc;
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
#define Y3B_FWD(N, T) recoupled_forward_kernel<kFeatures, N, T>
  Y3B_REC_DISPATCH(Y3B_FWD, per_atom, na, atom_count, s, rt, A, species, weights, species_count, energy, features,
                   status)
#undef Y3B_FWD
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
  int na = 1, th = 256;
  if (int rc = launch_shape(t, na, th)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && species && contraction_weights && energy && dEdA && species_count > 0,
                "null pointer argument");
  const size_t per_atom = grad_smem_per_atom(t.row_width, t.max_pass_components);
  const RecTabs rt = device_view(t);
  cudaStream_t s = as_stream(stream);
#define Y3B_GRAD(N, T) recoupled_energy_grad_kernel<N, T>
  Y3B_REC_DISPATCH(Y3B_GRAD, per_atom, na, atom_count, s, rt, A, species, contraction_weights, species_count,
                   energy, dEdA, status)
#undef Y3B_GRAD
}

namespace {

int check_sym_tables(const y3b_recoupled_sym_tables* tables) {
  Y3B_CHECK_ARG(tables != nullptr, "null tables");
  const y3b_recoupled_sym_tables& t = *tables;
  Y3B_CHECK_ARG(t.pass_count >= 1 && t.pass_count <= 64, "pass_count must be in [1, 64]");
  Y3B_CHECK_ARG(t.row_width >= 1 && t.row_width <= 4096, "row_width must be in [1, 4096]");
  Y3B_CHECK_ARG(t.max_pass_components >= 1 && t.dot_count >= 1, "empty recoupled tables");
  Y3B_CHECK_ARG(t.component_count >= 1 && t.cg_count >= 0 && t.own_count >= 0 && t.bp_count >= 0,
                "negative table sizes");
  Y3B_CHECK_ARG(t.pass_begin && t.comp && t.own && t.bp_begin && t.bp_gi && t.bp_other && t.bp_value &&
                    t.mirror && t.dot_begin && t.dot && (t.cg_count == 0 || (t.cg_index && t.cg_value)),
                "null table pointer");
  Y3B_CHECK_ARG(reinterpret_cast<uintptr_t>(t.comp) % 16 == 0 && reinterpret_cast<uintptr_t>(t.dot) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(t.own) % 8 == 0,
                "comp and dot must be 16-byte and own 8-byte aligned");
  return Y3B_OK;
}

}  // namespace

extern "C" int y3b_ace_recoupled_energy_grad_symmetric(const y3b_recoupled_sym_tables* tables, const void* A,
                                                       int64_t atom_count, const int32_t* species,
                                                       const double* contraction_weights, int64_t species_count,
                                                       double* energy, void* dEdA, int32_t* status, void* stream) {
  if (int rc = check_sym_tables(tables)) return rc;
  const y3b_recoupled_sym_tables& t = *tables;
  int na = 1, th = 256;
  if (int rc = launch_shape(t, na, th)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && species && contraction_weights && energy && dEdA && species_count > 0,
                "null pointer argument");
  const size_t per_atom = grad_smem_per_atom(t.row_width, t.max_pass_components);
  const SymTabs rt = sym_view(t);
  cudaStream_t s = as_stream(stream);
#define Y3B_SGRAD(N, T) recoupled_sym_energy_grad_kernel<N, T>
  Y3B_REC_DISPATCH(Y3B_SGRAD, per_atom, na, atom_count, s, rt, A, species, contraction_weights, species_count,
                   energy, dEdA, status)
#undef Y3B_SGRAD
}

extern "C" int y3b_ace_recoupled_energy_symmetric(const y3b_recoupled_sym_tables* tables, const void* A,
                                                  int64_t atom_count, const int32_t* species,
                                                  const double* contraction_weights, int64_t species_count,
                                                  double* energy, int32_t* status, void* stream) {
  if (int rc = check_sym_tables(tables)) return rc;
  const y3b_recoupled_sym_tables& t = *tables;
  int na = 1, th = 256;
  if (int rc = launch_shape(t, na, th)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && species && contraction_weights && energy && species_count > 0, "null pointer argument");
  const size_t per_atom = size_t(int64_t(t.row_width) + int64_t(t.max_pass_components)) * sizeof(double2);
  const SymTabs rt = sym_view(t);
  cudaStream_t s = as_stream(stream);
#define Y3B_SENER(N, T) recoupled_sym_energy_kernel<N, T>
  Y3B_REC_DISPATCH(Y3B_SENER, per_atom, na, atom_count, s, rt, A, species, contraction_weights, species_count,
                   energy, nullptr, status)
#undef Y3B_SENER
}

namespace {

int check_tile_tables(const y3b_recoupled_sym_tables& t, const y3b_recoupled_tile_tables* tiles) {
  Y3B_CHECK_ARG(tiles != nullptr, "null tile tables");
  const y3b_recoupled_tile_tables& u = *tiles;
  Y3B_CHECK_ARG(u.rows == 8, "tile rows must be 8");
  Y3B_CHECK_ARG(u.pass_count == t.pass_count, "tile tables cover %d passes, the symmetric tables %d", u.pass_count,
                t.pass_count);
  Y3B_CHECK_ARG(t.pass_count <= kTiledMaxLM1, "the tiled pass covers intermediate L up to %d", kTiledMaxLM1 - 1);
  Y3B_CHECK_ARG(u.tile_count >= 0 && u.step_count >= 0, "negative tile table sizes");
  Y3B_CHECK_ARG(u.tile_begin && u.tile_row && u.tile_col_begin && (u.step_count == 0 || (u.col_comp && u.kval)) &&
                    u.unit_begin && u.fix_begin && (u.unit_count == 0 || u.unit) && (u.fix_count == 0 || u.fix),
                "null tile table pointer");
  Y3B_CHECK_ARG(reinterpret_cast<uintptr_t>(u.unit) % 16 == 0 && reinterpret_cast<uintptr_t>(u.fix) % 16 == 0,
                "unit and fix must be 16-byte aligned");
  Y3B_CHECK_ARG(reinterpret_cast<uintptr_t>(u.col_comp) % 16 == 0 && reinterpret_cast<uintptr_t>(u.kval) % 16 == 0,
                "col_comp and kval must be 16-byte aligned");
  return Y3B_OK;
}

}  // namespace

extern "C" int y3b_ace_recoupled_energy_grad_tiled(const y3b_recoupled_sym_tables* tables,
                                                   const y3b_recoupled_tile_tables* tiles, const void* A,
                                                   int64_t atom_count, const int32_t* atom_order,
                                                   const int32_t* species, int64_t species_count, double* energy,
                                                   void* dEdA, int32_t* status, void* stream) {
  if (int rc = check_sym_tables(tables)) return rc;
  const y3b_recoupled_sym_tables& t = *tables;
  if (int rc = check_tile_tables(t, tiles)) return rc;
  const int th = t.threads_per_cta == 0 ? 256 : t.threads_per_cta;
  Y3B_CHECK_ARG(th == 256 || th == 512, "threads_per_cta must be 0 (256), 256 or 512");
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && species && energy && dEdA && species_count > 0, "null pointer argument");
  const int na = 32 / tiles->rows;
  const size_t per_atom = grad_smem_per_atom(t.row_width, t.max_pass_components);
  const SymTabs rt = sym_view(t);
  const TileTabs tt = tile_view(*tiles);
  Y3B_CHECK_ARG(tiles->scratch_slots >= 0 && tiles->scratch_slots <= 64, "scratch_slots must be in [0, 64]");
  const size_t smem = per_atom * size_t(na) + size_t(th / 32) * kTileStages * kStageBytes +
                      size_t(tiles->scratch_slots) * 512;
  Y3B_CHECK_ARG(smem <= 224 * 1024,
                "tiled recoupled pass needs %lld bytes of shared memory for %d atoms per CTA (max 224 KB)",
                (long long)smem, na);
  const int64_t groups = (atom_count + na - 1) / na;
  const int64_t grid = std::min<int64_t>(groups, int64_t(kSMs) * 64);
  cudaStream_t s = as_stream(stream);
  const double2* Ad = static_cast<const double2*>(A);
  double2* Gd = static_cast<double2*>(dEdA);
#define Y3B_TILED_LAUNCH(NA, TH)                                                                         \
  {                                                                                                      \
    auto kernel = recoupled_sym_tiled_grad_kernel<NA, TH>;                                               \
    Y3B_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));  \
    kernel<<<int(grid), TH, smem, s>>>(rt, tt, Ad, atom_count, atom_order, species, species_count, energy, \
                                       Gd, status);                                                      \
    Y3B_LAUNCH_CHECK();                                                                                  \
    return Y3B_OK;                                                                                       \
  }
  if (th == 256) Y3B_TILED_LAUNCH(4, 256)
  Y3B_TILED_LAUNCH(4, 512)
#undef Y3B_TILED_LAUNCH
}
