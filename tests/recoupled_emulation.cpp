// CPU emulation harness for the recoupled device passes (test infrastructure).
//
// Compiles ye3t_b200/csrc/recoupled_kernels.cuh as host C++ and runs a kernel
// as one CTA of 256 or 512 OS threads: __syncthreads is a std::barrier over
// the block, __shfl_xor_sync / __shfl_sync an exchange through a per-warp buffer between two
// warp barriers, __shared__ arrays are function statics and the dynamic shared
// memory one static buffer.  One CTA (gridDim.x = 1) walks every atom group, as
// the grid-stride loop of the kernels allows, so the emulated run follows the
// same source, barriers and index checks as the device run.
#define Y3B_EMULATE 1

#include <algorithm>
#include <atomic>
#include <barrier>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

struct double2 {
  double x, y;
};
struct int2 {
  int x, y;
};
struct int4 {
  int x, y, z, w;
};
inline double2 make_double2(double x, double y) { return double2{x, y}; }
inline int4 make_int4(int x, int y, int z, int w) { return int4{x, y, z, w}; }
struct Dim3 {
  unsigned x = 0, y = 0, z = 0;
};

static thread_local Dim3 threadIdx;
static thread_local Dim3 blockIdx;
static Dim3 gridDim;
static Dim3 blockDim;
alignas(16) static unsigned char y3b_emulated_smem[256 * 1024];
static std::barrier<>* g_block = nullptr;
static std::barrier<>* g_warp[32];
static double g_lanes[32][32];

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __launch_bounds__(...)
#define __restrict__
#define __shared__ static
#define __syncthreads() g_block->arrive_and_wait()
#define __syncwarp(...) g_warp[int(threadIdx.x) >> 5]->arrive_and_wait()

template <typename T>
inline T __ldg(const T* p) {
  return *p;
}
inline int atomicOr(int32_t* p, int v) { return __atomic_fetch_or(p, v, __ATOMIC_SEQ_CST); }
inline double __hiloint2double(int hi, int lo) {
  const uint64_t bits = (uint64_t(uint32_t(hi)) << 32) | uint64_t(uint32_t(lo));
  double d;
  std::memcpy(&d, &bits, sizeof d);
  return d;
}
inline double __shfl_xor_sync(unsigned, double v, int lane_mask) {
  const int w = int(threadIdx.x) >> 5, lane = int(threadIdx.x) & 31;
  g_lanes[w][lane] = v;
  g_warp[w]->arrive_and_wait();
  const double r = g_lanes[w][lane ^ lane_mask];
  g_warp[w]->arrive_and_wait();
  return r;
}
inline double __shfl_sync(unsigned, double v, int src_lane) {
  const int w = int(threadIdx.x) >> 5, lane = int(threadIdx.x) & 31;
  g_lanes[w][lane] = v;
  g_warp[w]->arrive_and_wait();
  const double r = g_lanes[w][src_lane & 31];
  g_warp[w]->arrive_and_wait();
  return r;
}
using std::fma;
using std::max;
using std::min;

#include "recoupled_kernels.cuh"

namespace {

template <typename F>
void run_block(int T, F body) {
  std::barrier<> block(T);
  std::vector<std::barrier<>*> warps;
  for (int w = 0; w < T / 32; ++w) warps.push_back(new std::barrier<>(32));
  g_block = &block;
  for (int w = 0; w < T / 32; ++w) g_warp[w] = warps[w];
  gridDim.x = 1;
  blockDim.x = T;
  std::vector<std::thread> threads;
  for (int i = 0; i < T; ++i)
    threads.emplace_back([i, &body] {
      threadIdx.x = unsigned(i);
      blockIdx.x = 0;
      body();
    });
  for (auto& t : threads) t.join();
  for (auto* w : warps) delete w;
  g_block = nullptr;
}

}  // namespace

#define EMU_SHAPES(CALL)                       \
  switch (na * 1000 + th) {                    \
    case 1256: CALL(1, 256); break;            \
    case 2256: CALL(2, 256); break;            \
    case 3256: CALL(3, 256); break;            \
    case 4256: CALL(4, 256); break;            \
    case 1512: CALL(1, 512); break;            \
    case 2512: CALL(2, 512); break;            \
    case 3512: CALL(3, 512); break;            \
    case 4512: CALL(4, 512); break;            \
    default: return -1;                        \
  }

extern "C" int emu_recoupled_energy_grad(int na, int th, const y3b_recoupled_tables* tables, const double* A,
                                         int64_t atom_count, const int32_t* species, const double* k,
                                         int64_t species_count, double* energy, double* G, int32_t* status) {
  const y3b::RecTabs t = y3b::device_view(*tables);
  const size_t smem = size_t(na) * size_t(2 * t.row_width + 2 * std::max(t.row_width, t.max_pass_components)) * 16;
  if (smem > sizeof(y3b_emulated_smem)) return -1;
  const auto* a2 = reinterpret_cast<const double2*>(A);
  auto* g2 = reinterpret_cast<double2*>(G);
#define EMU_GRAD(N, T)                                                                                        \
  run_block(T, [&] {                                                                                          \
    y3b::recoupled_energy_grad_kernel<N, T>(t, a2, atom_count, species, k, species_count, energy, g2, status); \
  })
  EMU_SHAPES(EMU_GRAD)
#undef EMU_GRAD
  return 0;
}

extern "C" int emu_recoupled_forward(int na, int th, int features_out, const y3b_recoupled_tables* tables,
                                     const double* A, int64_t atom_count, const int32_t* species, const double* k,
                                     int64_t species_count, double* energy, double* F, int32_t* status) {
  const y3b::RecTabs t = y3b::device_view(*tables);
  const size_t smem = size_t(na) * size_t(t.row_width + t.max_pass_components) * 16;
  if (smem > sizeof(y3b_emulated_smem)) return -1;
  const auto* a2 = reinterpret_cast<const double2*>(A);
  auto* f2 = reinterpret_cast<double2*>(F);
#define EMU_FEAT(N, T)                                                                                          \
  run_block(T, [&] {                                                                                            \
    y3b::recoupled_forward_kernel<true, N, T>(t, a2, atom_count, species, k, species_count, energy, f2, status); \
  })
#define EMU_ENER(N, T)                                                                                           \
  run_block(T, [&] {                                                                                             \
    y3b::recoupled_forward_kernel<false, N, T>(t, a2, atom_count, species, k, species_count, energy, f2, status); \
  })
  if (features_out) {
    EMU_SHAPES(EMU_FEAT)
  } else {
    EMU_SHAPES(EMU_ENER)
  }
#undef EMU_FEAT
#undef EMU_ENER
  return 0;
}

// The library's entry points under their own names and C signatures, running the
// emulated kernels on host memory: the Python wrapper (ye3t_b200.recoupling.
// RecoupledEvaluator) can be driven through its real ctypes bindings on CPU
// tensors.  The CTA shape comes from the tables as in the library.
namespace {
const char* g_error = "";
int emu_shape(const y3b_recoupled_tables* t, int& na, int& th) {
  if (t == nullptr) {
    g_error = "null tables";
    return -1;
  }
  na = t->atoms_per_cta == 0 ? 1 : t->atoms_per_cta;
  th = t->threads_per_cta == 0 ? 256 : t->threads_per_cta;
  if (na < 1 || na > 4 || (th != 256 && th != 512)) {
    g_error = "bad CTA shape";
    return -1;
  }
  return 0;
}
}  // namespace

extern "C" const char* y3b_last_error(void) { return g_error; }

extern "C" int y3b_ace_recoupled_energy_grad(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count,
                                             const int32_t* species, const double* contraction_weights,
                                             int64_t species_count, double* energy, void* dEdA, int32_t* status,
                                             void*) {
  int na = 1, th = 256;
  if (emu_shape(tables, na, th)) return -1;
  return emu_recoupled_energy_grad(na, th, tables, static_cast<const double*>(A), atom_count, species,
                                   contraction_weights, species_count, energy, static_cast<double*>(dEdA), status);
}

extern "C" int y3b_ace_recoupled_energy(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count,
                                        const int32_t* species, const double* contraction_weights,
                                        int64_t species_count, double* energy, int32_t* status, void*) {
  int na = 1, th = 256;
  if (emu_shape(tables, na, th)) return -1;
  return emu_recoupled_forward(na, th, 0, tables, static_cast<const double*>(A), atom_count, species,
                               contraction_weights, species_count, energy, nullptr, status);
}

extern "C" int y3b_ace_recoupled_features(const y3b_recoupled_tables* tables, const void* A, int64_t atom_count,
                                          void* features, int32_t* status, void*) {
  int na = 1, th = 256;
  if (emu_shape(tables, na, th)) return -1;
  return emu_recoupled_forward(na, th, 1, tables, static_cast<const double*>(A), atom_count, nullptr, nullptr, 0,
                               nullptr, static_cast<double*>(features), status);
}

// Symmetric passes (physical densities).
extern "C" int y3b_ace_recoupled_energy_grad_symmetric(const y3b_recoupled_sym_tables* tables, const void* A,
                                                       int64_t atom_count, const int32_t* species,
                                                       const double* k, int64_t species_count, double* energy,
                                                       void* dEdA, int32_t* status, void*) {
  int na = 1, th = 256;
  if (tables == nullptr) return -1;
  na = tables->atoms_per_cta == 0 ? 1 : tables->atoms_per_cta;
  th = tables->threads_per_cta == 0 ? 256 : tables->threads_per_cta;
  const y3b::SymTabs t = y3b::sym_view(*tables);
  const size_t smem = size_t(na) * size_t(2 * t.row_width + 2 * std::max(t.row_width, t.max_pass_components)) * 16;
  if (smem > sizeof(y3b_emulated_smem)) return -1;
  const auto* a2 = static_cast<const double2*>(A);
  auto* g2 = static_cast<double2*>(dEdA);
#define EMU_SGRAD(N, T)                                                                                            \
  run_block(T, [&] {                                                                                               \
    y3b::recoupled_sym_energy_grad_kernel<N, T>(t, a2, atom_count, species, k, species_count, energy, g2, status); \
  })
  EMU_SHAPES(EMU_SGRAD)
#undef EMU_SGRAD
  return 0;
}

extern "C" int y3b_ace_recoupled_energy_symmetric(const y3b_recoupled_sym_tables* tables, const void* A,
                                                  int64_t atom_count, const int32_t* species, const double* k,
                                                  int64_t species_count, double* energy, int32_t* status, void*) {
  int na = 1, th = 256;
  if (tables == nullptr) return -1;
  na = tables->atoms_per_cta == 0 ? 1 : tables->atoms_per_cta;
  th = tables->threads_per_cta == 0 ? 256 : tables->threads_per_cta;
  const y3b::SymTabs t = y3b::sym_view(*tables);
  const size_t smem = size_t(na) * size_t(t.row_width + t.max_pass_components) * 16;
  if (smem > sizeof(y3b_emulated_smem)) return -1;
  const auto* a2 = static_cast<const double2*>(A);
#define EMU_SENER(N, T)                                                                                          \
  run_block(T, [&] {                                                                                             \
    y3b::recoupled_sym_energy_kernel<N, T>(t, a2, atom_count, species, k, species_count, energy, nullptr, status); \
  })
  EMU_SHAPES(EMU_SENER)
#undef EMU_SENER
  return 0;
}

// Tiled symmetric adjoint: a CTA of 32 / rows atoms.
extern "C" int y3b_ace_recoupled_energy_grad_tiled(const y3b_recoupled_sym_tables* tables,
                                                   const y3b_recoupled_tile_tables* tiles, const void* A,
                                                   int64_t atom_count, const int32_t* order, const int32_t* species,
                                                   int64_t species_count, double* energy, void* dEdA,
                                                   int32_t* status, void*) {
  if (tables == nullptr || tiles == nullptr || tiles->rows != 8) return -1;
  const int th = tables->threads_per_cta == 0 ? 256 : tables->threads_per_cta;
  const int na = 32 / tiles->rows;
  const y3b::SymTabs t = y3b::sym_view(*tables);
  const y3b::TileTabs tt = y3b::tile_view(*tiles);
  const size_t smem = size_t(na) * size_t(2 * t.row_width + 2 * std::max(t.row_width, t.max_pass_components)) * 16 +
                     size_t(th / 32) * y3b::kTileStages * y3b::kStageBytes + size_t(tiles->scratch_slots) * 512;
  if (smem > sizeof(y3b_emulated_smem)) return -1;
  const auto* a2 = static_cast<const double2*>(A);
  auto* g2 = static_cast<double2*>(dEdA);
#define EMU_TGRAD(N, T)                                                                                           \
  run_block(T, [&] {                                                                                              \
    y3b::recoupled_sym_tiled_grad_kernel<N, T>(t, tt, a2, atom_count, order, species, species_count, energy, g2,  \
                                               status);                                                           \
  })
  if (na == 4 && th == 256) EMU_TGRAD(4, 256);
  else if (na == 4 && th == 512) EMU_TGRAD(4, 512);
  else return -1;
#undef EMU_TGRAD
  return 0;
}
