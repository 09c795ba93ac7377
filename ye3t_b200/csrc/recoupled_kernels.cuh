// Device code of the recoupled passes (see recoupled.cu for what they
// compute).  Compiled by nvcc through recoupled.cu; with Y3B_EMULATE defined
// it also compiles as host C++ for the CPU emulation harness of the tests,
// which runs one OS thread per CUDA thread with std::barrier as the block
// barrier, so that this exact source is checked against the oracle without a
// GPU.
#pragma once

#include <stdint.h>

#include <cstring>

#include "ye3t_b200.h"

#ifdef Y3B_EMULATE
#define Y3B_DYNAMIC_SMEM(T, name) T* name = reinterpret_cast<T*>(y3b_emulated_smem)
#else
#define Y3B_DYNAMIC_SMEM(T, name) extern __shared__ T name[]
#endif

namespace y3b {
namespace {


__host__ __device__ inline double2 rmul(double2 a, double2 b) {
  return make_double2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// 16-byte asynchronous global-to-shared copies (cp.async, completion tracked
// per thread in commit groups).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
#ifdef Y3B_EMULATE
  std::memcpy(smem_dst, gmem_src, 16);
#else
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem_src) : "memory");
#endif
}
__device__ __forceinline__ void cp_async_commit() {
#ifndef Y3B_EMULATE
  asm volatile("cp.async.commit_group;\n" ::: "memory");
#endif
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
#ifndef Y3B_EMULATE
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
#endif
}

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

inline RecTabs device_view(const y3b_recoupled_tables& t) {
  return RecTabs{t.pass_count, t.max_pass_components, t.row_width, t.dot_count,
                 t.component_count, t.cg_count, t.own_count, t.bp_count,
                 t.pass_begin, reinterpret_cast<const int4*>(t.comp), t.cg_index, t.cg_value,
                 reinterpret_cast<const int2*>(t.own), t.bp_begin, t.bp_gi, t.bp_other, t.bp_value,
                 t.feature_count, t.feat_count, t.dot_begin, reinterpret_cast<const int4*>(t.dot), t.feat_index,
                 t.feat_weight};
}

// Fixed-order block sum of one double per thread (warp shuffles, then the
// warps in order); the result is valid in thread 0.
template <int TH>
__device__ __forceinline__ double block_sum(double v, double* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  double s = 0.0;
  if (threadIdx.x == 0)
    for (int w = 0; w < TH / 32; ++w) s += red[w];
  return s;
}

// Tables of the symmetric passes (physical densities, M >= 0 components only).
struct SymTabs {
  int32_t pass_count, max_pass_components, row_width, dot_count;
  int64_t component_count, cg_count, own_count, bp_count;
  const int32_t* pass_begin;
  const int4* comp;  // (a, b, cg_begin, cg_count), (M, own_begin, own_count, (-1)^p)
  const int32_t* cg_index;
  const double* cg_value;
  const int2* own;  // (partner's M = 0 local component, contraction)
  const int32_t* bp_begin;
  const int32_t* bp_gi;  // 2 * component + (1: conj(gI) of a negative M)
  const int32_t* bp_other;
  const double* bp_value;
  const int32_t* mirror;  // 2 * (entry of -m) + (m & 1) for an entry of negative m, else -1
  const int32_t* dot_begin;
  const int4* dot;  // (A's M = 0 local component, B's, (-1)^p_B, 0)
};

inline SymTabs sym_view(const y3b_recoupled_sym_tables& t) {
  return SymTabs{t.pass_count, t.max_pass_components, t.row_width, t.dot_count,
                 t.component_count, t.cg_count, t.own_count, t.bp_count,
                 t.pass_begin, reinterpret_cast<const int4*>(t.comp), t.cg_index, t.cg_value,
                 reinterpret_cast<const int2*>(t.own), t.bp_begin, t.bp_gi, t.bp_other, t.bp_value,
                 t.mirror, t.dot_begin, reinterpret_cast<const int4*>(t.dot)};
}

// Shared-memory arrays hold NA atoms side by side: entry e of atom a at
// [e * NA + a].  A CTA takes atoms [g NA, g NA + NA); every table entry it
// loads (coupling term, contraction-list entry, back-propagation entry,
// contraction) serves all NA atoms, and the NA sums are independent chains.
template <int NA, int TH, typename Tabs>
__device__ __forceinline__ void build_components(const Tabs& t, const double2* sA, double2* sI, int c0, int nc,
                                                 int W, bool& bad) {
  for (int c = threadIdx.x; c < nc; c += TH) {
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
          const double2 p = rmul(sA[ia * NA + a], sA[ib * NA + a]);
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
template <int NA, int TH>
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
  for (int i = threadIdx.x; i < W * NA; i += TH) {
    const int a = i % NA, e = i / NA;
    sA[i] = a < nv ? A[(first + a) * W + e] : make_double2(0.0, 0.0);
    if (sGA != nullptr) sGA[i] = make_double2(0.0, 0.0);
  }
  return nv;
}

template <int NA, int TH>
__global__ void __launch_bounds__(TH)
recoupled_energy_grad_kernel(RecTabs t, const double2* __restrict__ A, int64_t atom_count,
                             const int32_t* __restrict__ species, const double* __restrict__ k,
                             int64_t species_count, double* __restrict__ energy, double2* __restrict__ G,
                             int32_t* status) {
  Y3B_DYNAMIC_SMEM(double2, rec_smem);
  __shared__ double red[TH / 32];
  const int W = t.row_width;
  const int maxc = t.max_pass_components;
  // the component regions also stage step 3's parts (at least W entries per atom)
  const int cw = maxc > W ? maxc : W;
  double2* sA = rec_smem;          // [W][NA] the atoms' A rows
  double2* sGA = sA + W * NA;      // [W][NA] dE/dA of the rows
  double2* sI = sGA + W * NA;      // [cw][NA] components of the pass
  double2* sG = sI + cw * NA;      // [cw][NA] their adjoints
  const int tid = threadIdx.x;
  const int64_t groups = (atom_count + NA - 1) / NA;
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t first = grp * NA;
    const double* kz[NA];
    const int nv = load_atoms<NA, TH>(first, atom_count, W, A, species, k, species_count, t.dot_count, sA, sGA, kz,
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
      build_components<NA, TH>(t, sA, sI, c0, nc, W, bad);
      __syncthreads();
      // 2. adjoints of the components and the energy shares
      for (int c = tid; c < nc; c += TH) {
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
      // 3. back-propagation into the A rows.  Each entry's list is split into P
      //    parts when the block has at least two threads per entry (P threads per
      //    entry); the partial sums go to the component buffer, which step 2 no
      //    longer needs, and are added to the entry in part order.
      const int P = (2 * W <= TH && (TH / W) * W <= cw) ? TH / W : 1;  // uniform
      double2* part = sI;  // [P][W][NA]
      for (int u = tid; u < W * P; u += TH) {
        const int i = u % W, pi = u / W;
        const int64_t at = int64_t(L) * W + i;
        const int b0 = t.bp_begin[at], b1 = t.bp_begin[at + 1];
        double2 ga[NA];
#pragma unroll
        for (int a = 0; a < NA; ++a) ga[a] = make_double2(0.0, 0.0);
        if (b0 < 0 || b1 < b0 || int64_t(b1) > t.bp_count) {
          bad = true;
        } else {
          const int len = b1 - b0;
          const int q0 = b0 + (len * pi) / P, q1 = b0 + (len * (pi + 1)) / P;
          for (int q = q0; q < q1; ++q) {
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
              const double2 term = o < 0 ? g : rmul(g, sA[o * NA + a]);
              ga[a].x = fma(cv, term.x, ga[a].x);
              ga[a].y = fma(cv, term.y, ga[a].y);
            }
          }
        }
#pragma unroll
        for (int a = 0; a < NA; ++a) part[(pi * W + i) * NA + a] = ga[a];
      }
      __syncthreads();
      for (int u = tid; u < W * NA; u += TH) {
        double2 acc = sGA[u];
        for (int pi = 0; pi < P; ++pi) {
          const double2 v = part[pi * W * NA + u];
          acc.x += v.x;
          acc.y += v.y;
        }
        sGA[u] = acc;
      }
      __syncthreads();
    }
    if (bad && status) atomicOr(status, Y3B_STATUS_TABLE);
    for (int i = tid; i < W * NA; i += TH) {
      const int a = i % NA, e = i / NA;
      if (a < nv) G[(first + a) * W + e] = sGA[i];
    }
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      const double total = block_sum<TH>(ep[a], red);
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
template <bool kFeatures, int NA, int TH>
__global__ void __launch_bounds__(TH)
recoupled_forward_kernel(RecTabs t, const double2* __restrict__ A, int64_t atom_count,
                         const int32_t* __restrict__ species, const double* __restrict__ k, int64_t species_count,
                         double* __restrict__ energy, double2* __restrict__ features, int32_t* status) {
  Y3B_DYNAMIC_SMEM(double2, rec_smem);
  __shared__ double red[TH / 32];
  const int W = t.row_width;
  double2* sA = rec_smem;     // [W][NA]
  double2* sI = sA + W * NA;  // [max_pass_components][NA]
  const int tid = threadIdx.x;
  const int64_t groups = (atom_count + NA - 1) / NA;
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t first = grp * NA;
    const double* kz[NA];
    const int nv = load_atoms<NA, TH>(first, atom_count, W, A, kFeatures ? nullptr : species, kFeatures ? nullptr : k,
                                  species_count, t.dot_count, sA, nullptr, kz, status);
    if constexpr (kFeatures) {
      for (int64_t i = tid; i < int64_t(nv) * t.feature_count; i += TH)
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
      build_components<NA, TH>(t, sA, sI, c0, nc, W, bad);
      __syncthreads();
      for (int j = tid; j < nd; j += TH) {
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
            const double2 p = rmul(sI[(q.x + m) * NA + a], sI[(q.y + 2 * L - m) * NA + a]);
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
        const double total = block_sum<TH>(ep[a], red);
        if (tid == 0 && a < nv) energy[first + a] = total;
        __syncthreads();
      }
    } else {
      __syncthreads();
    }
  }
}

// Symmetric adjoint (physical densities): per L the M >= 0 components, their
// adjoints gI[M] = (-1)^p conj(sum_q k[d_q] I_partner[M]), the energy
// 1/2 Re(I[0] gI[0]) + sum_{M>0} Re(I[M] gI[M]), and the back-propagation into
// the m >= 0 half of each A row (entries of a negative M read conj(gI)); the
// m < 0 half is mirrored at the end, G[-m] = (-1)^m conj(G[m]).
template <int NA, int TH>
__global__ void __launch_bounds__(TH)
recoupled_sym_energy_grad_kernel(SymTabs t, const double2* __restrict__ A, int64_t atom_count,
                                 const int32_t* __restrict__ species, const double* __restrict__ k,
                                 int64_t species_count, double* __restrict__ energy, double2* __restrict__ G,
                                 int32_t* status) {
  Y3B_DYNAMIC_SMEM(double2, rec_smem);
  __shared__ double red[TH / 32];
  const int W = t.row_width;
  const int maxc = t.max_pass_components;
  const int cw = maxc > W ? maxc : W;  // the component regions also stage step 3's parts
  double2* sA = rec_smem;
  double2* sGA = sA + W * NA;
  double2* sI = sGA + W * NA;
  double2* sG = sI + cw * NA;
  const int tid = threadIdx.x;
  const int64_t groups = (atom_count + NA - 1) / NA;
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t first = grp * NA;
    const double* kz[NA];
    const int nv = load_atoms<NA, TH>(first, atom_count, W, A, species, k, species_count, t.dot_count, sA, sGA, kz,
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
        bad = true;  // uniform over the block
        continue;
      }
      build_components<NA, TH>(t, sA, sI, c0, nc, W, bad);
      __syncthreads();
      for (int c = tid; c < nc; c += TH) {
        const int4 d = __ldg(t.comp + 2 * (c0 + c) + 1);  // (M, own_begin, own_count, sign)
        double2 acc[NA];
#pragma unroll
        for (int a = 0; a < NA; ++a) acc[a] = make_double2(0.0, 0.0);
        if (d.y < 0 || d.z < 0 || int64_t(d.y) + d.z > t.own_count) {
          bad = true;
        } else {
          for (int q = d.y; q < d.y + d.z; ++q) {
            const int2 e = __ldg(t.own + q);
            const int p = e.x + d.x;
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
        const double sg = d.w < 0 ? -1.0 : 1.0;
        const double wm = d.x == 0 ? 0.5 : 1.0;
#pragma unroll
        for (int a = 0; a < NA; ++a) {
          const double2 g = make_double2(sg * acc[a].x, -sg * acc[a].y);
          sG[c * NA + a] = g;
          const double2 iv = sI[c * NA + a];
          ep[a] = fma(wm, iv.x * g.x - iv.y * g.y, ep[a]);
        }
      }
      __syncthreads();
      const int P = (2 * W <= TH && (TH / W) * W <= cw) ? TH / W : 1;  // uniform
      double2* part = sI;  // [P][W][NA]; step 2 is done with sI
      for (int u = tid; u < W * P; u += TH) {
        const int i = u % W, pi = u / W;
        const int64_t at = int64_t(L) * W + i;
        const int b0 = t.bp_begin[at], b1 = t.bp_begin[at + 1];
        double2 ga[NA];
#pragma unroll
        for (int a = 0; a < NA; ++a) ga[a] = make_double2(0.0, 0.0);
        if (b0 < 0 || b1 < b0 || int64_t(b1) > t.bp_count) {
          bad = true;
        } else {
          const int len = b1 - b0;
          const int q0 = b0 + (len * pi) / P, q1 = b0 + (len * (pi + 1)) / P;
          for (int q = q0; q < q1; ++q) {
            const int code = __ldg(t.bp_gi + q);
            const int gi = code >> 1;
            const int o = __ldg(t.bp_other + q);
            if (code < 0 || gi >= nc || o >= W) {
              bad = true;
              continue;
            }
            const double cv = __ldg(t.bp_value + q);
#pragma unroll
            for (int a = 0; a < NA; ++a) {
              double2 g = sG[gi * NA + a];
              if (code & 1) g.y = -g.y;
              const double2 term = o < 0 ? g : rmul(g, sA[o * NA + a]);
              ga[a].x = fma(cv, term.x, ga[a].x);
              ga[a].y = fma(cv, term.y, ga[a].y);
            }
          }
        }
#pragma unroll
        for (int a = 0; a < NA; ++a) part[(pi * W + i) * NA + a] = ga[a];
      }
      __syncthreads();
      for (int u = tid; u < W * NA; u += TH) {
        double2 acc = sGA[u];
        for (int pi = 0; pi < P; ++pi) {
          const double2 v = part[pi * W * NA + u];
          acc.x += v.x;
          acc.y += v.y;
        }
        sGA[u] = acc;
      }
      __syncthreads();
    }
    // the m < 0 half of each row from the m > 0 half (sources and targets are disjoint)
    for (int u = tid; u < W * NA; u += TH) {
      const int i = u / NA, a = u % NA;
      const int mi = __ldg(t.mirror + i);
      if (mi < 0) continue;
      const int src = mi >> 1;
      if (src >= W) {
        bad = true;
        continue;
      }
      const double2 v = sGA[src * NA + a];
      const double sg = (mi & 1) ? -1.0 : 1.0;
      sGA[u] = make_double2(sg * v.x, -sg * v.y);
    }
    __syncthreads();
    if (bad && status) atomicOr(status, Y3B_STATUS_TABLE);
    for (int i = tid; i < W * NA; i += TH) {
      const int a = i % NA, e = i / NA;
      if (a < nv) G[(first + a) * W + e] = sGA[i];
    }
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      const double total = block_sum<TH>(ep[a], red);
      if (tid == 0 && a < nv) energy[first + a] = total;
      __syncthreads();
    }
  }
}

// Symmetric forward energy: T_d = (-1)^p_B (Re(I_A[0] conj(I_B[0])) +
// 2 sum_{M>0} Re(I_A[M] conj(I_B[M]))), e = sum_d k[z, d] T_d.
template <int NA, int TH>
__global__ void __launch_bounds__(TH)
recoupled_sym_energy_kernel(SymTabs t, const double2* __restrict__ A, int64_t atom_count,
                            const int32_t* __restrict__ species, const double* __restrict__ k, int64_t species_count,
                            double* __restrict__ energy, double2* __restrict__ unused, int32_t* status) {
  Y3B_DYNAMIC_SMEM(double2, rec_smem);
  __shared__ double red[TH / 32];
  const int W = t.row_width;
  double2* sA = rec_smem;
  double2* sI = sA + W * NA;
  const int tid = threadIdx.x;
  const int64_t groups = (atom_count + NA - 1) / NA;
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t first = grp * NA;
    const double* kz[NA];
    const int nv = load_atoms<NA, TH>(first, atom_count, W, A, species, k, species_count, t.dot_count, sA, nullptr,
                                      kz, status);
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
      build_components<NA, TH>(t, sA, sI, c0, nc, W, bad);
      __syncthreads();
      for (int j = tid; j < nd; j += TH) {
        const int4 q = __ldg(t.dot + d0 + j);
        if (q.x < 0 || q.y < 0 || q.x + L >= nc || q.y + L >= nc) {
          bad = true;
          continue;
        }
        double T[NA];
#pragma unroll
        for (int a = 0; a < NA; ++a) T[a] = 0.0;
        for (int m = 0; m <= L; ++m) {
          const double w = m == 0 ? 1.0 : 2.0;
#pragma unroll
          for (int a = 0; a < NA; ++a) {
            const double2 x = sI[(q.x + m) * NA + a], y = sI[(q.y + m) * NA + a];
            T[a] = fma(w, fma(x.x, y.x, x.y * y.y), T[a]);
          }
        }
        const double sg = q.z < 0 ? -1.0 : 1.0;
#pragma unroll
        for (int a = 0; a < NA; ++a) ep[a] = fma(__ldg(kz[a] + d0 + j), sg * T[a], ep[a]);
      }
      __syncthreads();
    }
    if (bad && status) atomicOr(status, Y3B_STATUS_TABLE);
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      const double total = block_sum<TH>(ep[a], red);
      if (tid == 0 && a < nv) energy[first + a] = total;
      __syncthreads();
    }
  }
}

// Dense tiles of the symmetric pass's contraction weights (RecoupledTiles).
struct TileTabs {
  int32_t rows, pass_count;
  int64_t tile_count, step_count, item_count, group_count, pack_count;
  const int32_t* tile_begin;
  const int32_t* tile_row;
  const int32_t* tile_col_begin;
  const int32_t* col_comp;
  const int32_t* bp_item_begin;
  const int32_t* t_item_begin;
  const int32_t* t_item;
  const int32_t* bp_group_begin;
  const int32_t* bp_group_off;
  const int4* bp_pack;
  int64_t unit_count, fix_count;
  int32_t scratch_slots;
  const int32_t* unit_begin;
  const int4* unit;
  const int32_t* fix_begin;
  const int4* fix;
  const double* kval;
};

inline TileTabs tile_view(const y3b_recoupled_tile_tables& t) {
  return TileTabs{t.rows, t.pass_count, t.tile_count, t.step_count, t.item_count, t.group_count, t.pack_count,
                  t.tile_begin, t.tile_row, t.tile_col_begin, t.col_comp, t.bp_item_begin, t.t_item_begin,
                  t.t_item, t.bp_group_begin, t.bp_group_off, reinterpret_cast<const int4*>(t.bp_pack),
                  t.unit_count, t.fix_count, t.scratch_slots, t.unit_begin, reinterpret_cast<const int4*>(t.unit),
                  t.fix_begin, reinterpret_cast<const int4*>(t.fix), t.kval};
}

// Step 1 of the tiled adjoint with lanes as (component, atom): a warp builds
// 32 / NA consecutive components for its NA atoms at a time, so each table
// entry it loads serves NA lanes and its A-row reads are whole [entry][NA]
// rows.
template <int NA, int TH>
__device__ __forceinline__ void build_components_lanes(const SymTabs& t, const double2* sA, double2* sI, int c0,
                                                       int nc, int W, bool& bad) {
  constexpr int R = 32 / NA;
  constexpr int NW = TH / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int a = lane % NA;
  // the record of the lane's component in the warp's next group is loaded a group ahead
  int4 dn = make_int4(-1, 0, 0, 0);
  if (warp * R + lane / NA < nc) dn = __ldg(t.comp + 2 * (c0 + warp * R + lane / NA));
  for (int g = warp; g * R < nc; g += NW) {
    const int c = g * R + lane / NA;
    const int4 d = dn;
    if (c + NW * R < nc) dn = __ldg(t.comp + 2 * (c0 + c + NW * R));
    if (c >= nc) continue;
    double2 v = make_double2(d.x < 0 ? 1.0 : 0.0, 0.0);
    if (d.x < 0) {
    } else if (d.w == 0) {
      if (d.x < W)
        v = sA[d.x * NA + a];
      else
        bad = true;
    } else if (d.z < 0 || int64_t(d.z) + d.w > t.cg_count || d.y < 0) {
      bad = true;
    } else {
      for (int qb = d.z; qb < d.z + d.w; qb += 4) {  // four terms' table entries in flight
        int ix[4];
        double cv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const bool in = qb + u < d.z + d.w;
          ix[u] = in ? __ldg(t.cg_index + qb + u) : 0;
          cv[u] = in ? __ldg(t.cg_value + qb + u) : 0.0;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (qb + u >= d.z + d.w) break;
          const int ia = d.x + (ix[u] & 255), ib = d.y + (ix[u] >> 8);
          if (ia >= W || ib < 0 || ib >= W) {
            bad = true;
            continue;
          }
          const double2 p = rmul(sA[ia * NA + a], sA[ib * NA + a]);
          v.x = fma(cv[u], p.x, v.x);
          v.y = fma(cv[u], p.y, v.y);
        }
      }
    }
    sI[c * NA + a] = v;
  }
}

// Per-warp staging ring of step 2: each stage holds eight column steps (two
// k = 4 steps of the tile product) of the warp's current unit, their column
// offsets (32 bytes) and the weights of all rows (8 x 8 doubles) for the
// species of the CTA's first atom, copied from global memory kTileStages
// stages ahead of their use so that the weights' L2 latency overlaps the
// arithmetic.  A CTA whose atoms have several species reads each species'
// weights from global memory instead.
constexpr int kTileStages = 4;
constexpr int kStageSteps = 8;
constexpr int kStageBytes = 4 * kStageSteps + kStageSteps * 8 * 8;

// One FP64 tensor-core step D = A B + C of shape m8n8k4 (mma.sync: tcgen05 has
// no FP64 kind, so this is the FP64 matrix path of sm_100).  Fragments of lane
// l: a = A[l / 4][l % 4], b = B[l % 4][l / 4], (d0, d1) = C, D[l / 4][2 (l % 4)
// + {0, 1}].  The CPU emulation gathers the fragments through warp exchanges
// and forms each output as C + sum_k A[r][k] B[k][n] with fma in k order.
__device__ __forceinline__ void dmma_m8n8k4(double& d0, double& d1, double a, double b) {
#ifdef Y3B_EMULATE
  const int lane = threadIdx.x & 31, r = lane >> 2, tg = lane & 3;
  double av[4], b0[4], b1[4];
  for (int k = 0; k < 4; ++k) {
    av[k] = __shfl_sync(0xffffffffu, a, r * 4 + k);
    b0[k] = __shfl_sync(0xffffffffu, b, 4 * (2 * tg) + k);
    b1[k] = __shfl_sync(0xffffffffu, b, 4 * (2 * tg + 1) + k);
  }
  for (int k = 0; k < 4; ++k) {
    d0 = fma(av[k], b0[k], d0);
    d1 = fma(av[k], b1[k], d1);
  }
#else
  asm("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};\n"
      : "+d"(d0), "+d"(d1)
      : "d"(a), "d"(b));
#endif
}

// Column walk of one unit on the FP64 tensor cores.  Each stage of the ring is
// the k = 4 of one m8n8k4 step: acc[M] += K[8 rows, 4 steps] x I[4 steps, 8]
// for every M of the pass, where the 8 columns of I are (atom, real or
// imaginary part) of the column's component + M.  Lane l holds the weight
// K[row l / 4, step l % 4], the I value of step l % 4 for atom l / 8 (real
// part when l / 4 is even), and the sums of row l / 4 and atom l % 4 (real,
// imaginary) in acc[M].  STAGED: the CTA's one species' weights come from the
// ring; otherwise each species among the CTA's atoms takes its own step with
// its weights read from global memory and the I values of the other species'
// atoms set to zero.  Each lane reads its own column of the stage; one outside
// the pass sets bad and is replaced by column 0, so every read stays inside the
// component region.
template <bool STAGED, int LM1, int NA>
__device__ __forceinline__ void tile_walk_mma(const TileTabs& tt, int q0, int nq, int nc, const double* sId,
                                              const double* const (&kw)[NA], const int (&za)[NA],
                                              unsigned char* ring, double (&acc)[LM1][2], bool& bad) {
  constexpr int R = 8;
  const int lane = threadIdx.x & 31;
  const int kk = lane & 3, row = lane >> 2;
  const int ab = lane >> 3, part = (lane >> 2) & 1;  // the lane's I value: atom, real/imaginary
  const double* sIl = sId + ab * 2 + part;            // I[c + M] of this lane at sIl[2 NA (c + M)]
  const int lim = nc - LM1;                           // a column c needs c + LM1 <= nc
  const int ns = (nq + 1) >> 1;                       // stages of two quads
  int zb = za[0];
#pragma unroll
  for (int s = 1; s < NA; ++s)
    if (ab == s) zb = za[s];
  // the lane's share of a stage copy: 16 bytes of weights (lane < 16 for the
  // stage's first quad, lane >= 16 for its second), and lanes 0 / 1 the columns
  // of the first / second quad
  const int half = lane >> 4;
  const char* wsrc = reinterpret_cast<const char*>(kw[0] + 2 * lane);
  const char* csrc = reinterpret_cast<const char*>(tt.col_comp + q0 + 4 * (lane & 1));
  auto issue = [&](int Q) {  // stage Q: quads 2Q and 2Q + 1 (every lane commits a group)
    unsigned char* st = ring + (Q & (kTileStages - 1)) * kStageBytes;
    if (STAGED && 2 * Q + half < nq)
      cp_async16(st + 4 * kStageSteps + 16 * lane, wsrc + int64_t(Q) * (R * kStageSteps * 8));
    if (lane < 2 && 2 * Q + lane < nq) cp_async16(st + 16 * lane, csrc + int64_t(Q) * (4 * kStageSteps));
    cp_async_commit();
  };
  // one k = 4 step: quad h of the stage
  auto kstep = [&](const unsigned char* st, int Q, int h) {
    const int col = reinterpret_cast<const int*>(st)[4 * h + kk];
    // a column outside the pass sets bad and is replaced by column 0
    const bool ok = col >= 0 && col <= lim;
    bad = bad || !ok;
    const double* bI = sIl + (ok ? col : 0) * (2 * NA);
    if (STAGED) {
      const double av = reinterpret_cast<const double*>(st + 4 * kStageSteps)[(4 * h + kk) * R + row];
#pragma unroll
      for (int M = 0; M < LM1; ++M) dmma_m8n8k4(acc[M][0], acc[M][1], av, bI[2 * NA * M]);
    } else {
#pragma unroll
      for (int s = 0; s < NA; ++s) {
        bool first = true;
#pragma unroll
        for (int j = 0; j < s; ++j) first = first && za[j] != za[s];
        if (!first) continue;  // uniform over the warp
        const double av = __ldg(kw[s] + int64_t(R) * (kStageSteps * Q + 4 * h + kk) + row);
        const bool on = zb == za[s];
#pragma unroll
        for (int M = 0; M < LM1; ++M) dmma_m8n8k4(acc[M][0], acc[M][1], av, on ? bI[2 * NA * M] : 0.0);
      }
    }
  };
#pragma unroll
  for (int s = 0; s < kTileStages; ++s) issue(s);
  for (int Q = 0; Q < ns; ++Q) {
    cp_async_wait<kTileStages - 1>();
    __syncwarp();
    const unsigned char* st = ring + (Q & (kTileStages - 1)) * kStageBytes;
    kstep(st, Q, 0);
    if (2 * Q + 1 < nq) kstep(st, Q, 1);  // uniform over the warp
    __syncwarp();
    issue(Q + kTileStages);
  }
}

// Step 2 of the tiled symmetric adjoint for one pass of L = LM1 - 1 (tiles of
// 8 rows, NA = 4 atoms).  A warp takes a work unit (a tile, or a chunk of a
// long tile's columns; units ordered by decreasing length go to the warps in a
// snake order) and walks its columns on the FP64 tensor cores for all LM1
// components at once (tile_walk_mma), so that lane l ends with the sums of row
// l / 4 and atom l % 4.  A whole tile ends by writing gI = (-1)^p conj(acc)
// for its rows and adding the energy shares w_M Re(I gI) (w_0 = 1/2).  The
// first chunk of a cut tile leaves its sums in sG, each later chunk in its
// scratch slot, and after a barrier each cut tile's fix-up adds the later
// chunks in slot order and finishes as a whole tile does.  Every sum has a
// fixed order, so the results do not depend on which warp runs what.  A
// column, row or unit outside the pass is skipped and sets bad.
template <int LM1, int NA, int TH>
__device__ __forceinline__ void tiled_adjoint_pass(const SymTabs& t, const TileTabs& tt, int L, int c0, int nc,
                                                   const double2* sI, double2* sG, const double* const (&kw)[NA],
                                                   const int (&za)[NA], bool staged, unsigned char* ring,
                                                   double2* scratch, double& ep, bool& bad) {
  constexpr int R = 8;
  static_assert(NA == 4, "one m8n8k4 step holds 8 rows of 4 atoms");
  constexpr int SLOT = R * LM1 * NA;  // double2 per scratch slot
  constexpr int NW = TH / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int a = lane & 3, row = lane >> 2;
  const double* sId = reinterpret_cast<const double*>(sI);
  const int t0 = tt.tile_begin[L], t1 = tt.tile_begin[L + 1];
  const int u0 = tt.unit_begin[L], u1 = tt.unit_begin[L + 1];
  if (t0 < 0 || t1 < t0 || int64_t(t1) > tt.tile_count || u0 < 0 || u1 < u0 || int64_t(u1) > tt.unit_count) {
    bad = true;
    return;
  }
  // a whole tile's ending: gI and the energy shares from the lane's sums
  auto finish = [&](int tile, const double (&acc)[LM1][2]) {
    const int rowc = tt.tile_row[int64_t(tile) * R + row];
    if (rowc < -1 || rowc + LM1 > nc) {
      bad = true;
      return;
    }
    if (rowc < 0) return;
    const double sg = __ldg(t.comp + 2 * (c0 + rowc) + 1).w < 0 ? -1.0 : 1.0;
#pragma unroll
    for (int M = 0; M < LM1; ++M) {
      const double2 g = make_double2(sg * acc[M][0], -sg * acc[M][1]);
      sG[(rowc + M) * NA + a] = g;
      const double2 iv = sI[(rowc + M) * NA + a];
      ep = fma(M == 0 ? 0.5 : 1.0, iv.x * g.x - iv.y * g.y, ep);
    }
  };
  const int units = u1 - u0;
  for (int k = 0;; ++k) {
    const int item = (k & 1) ? k * NW + (NW - 1 - warp) : k * NW + warp;  // uniform over the warp
    if (item >= units) break;
    const int4 u = __ldg(tt.unit + u0 + item);  // (tile, first step, end step, kind)
    const int tile = u.x;
    if (tile < t0 || tile >= t1 || u.w < -2 || (u.w >= 0 && (u.w + 1) * LM1 > tt.scratch_slots)) {
      bad = true;
      continue;
    }
    const int q0 = tt.tile_col_begin[tile], q1 = tt.tile_col_begin[tile + 1];
    const int qs = q0 + u.y, qe = q0 + u.z;
    if (q0 < 0 || q1 < q0 || (q0 & 3) || u.y < 0 || u.z < u.y || ((u.z - u.y) & 3) || (u.y & 3) || qe > q1 ||
        int64_t(q1) > tt.step_count) {
      bad = true;
      continue;
    }
    double acc[LM1][2];
#pragma unroll
    for (int M = 0; M < LM1; ++M) acc[M][0] = acc[M][1] = 0.0;
    const double* kwu[NA];
#pragma unroll
    for (int s = 0; s < NA; ++s) kwu[s] = kw[s] + int64_t(R) * qs;
    if (staged)  // uniform over the CTA
      tile_walk_mma<true, LM1, NA>(tt, qs, (qe - qs) / 4, nc, sId, kwu, za, ring, acc, bad);
    else
      tile_walk_mma<false, LM1, NA>(tt, qs, (qe - qs) / 4, nc, sId, kwu, za, ring, acc, bad);
    if (u.w == -1) {
      finish(tile, acc);
    } else {
      const int rowc = tt.tile_row[int64_t(tile) * R + row];
      if (rowc < -1 || rowc + LM1 > nc) {
        bad = true;
      } else if (u.w == -2) {
        if (rowc >= 0) {
#pragma unroll
          for (int M = 0; M < LM1; ++M)
            sG[(rowc + M) * NA + a] = make_double2(acc[M][0], acc[M][1]);  // the first chunk's sums, unsigned
        }
      } else {
#pragma unroll
        for (int M = 0; M < LM1; ++M)
          scratch[u.w * SLOT + (row * LM1 + M) * NA + a] = make_double2(acc[M][0], acc[M][1]);
      }
    }
  }
  const int f0 = tt.fix_begin[L], f1 = tt.fix_begin[L + 1];
  if (f1 > f0) {  // uniform over the CTA
    __syncthreads();
    if (f0 < 0 || int64_t(f1) > tt.fix_count) {
      bad = true;
      return;
    }
    for (int f = f0 + warp; f < f1; f += NW) {
      const int4 fx = __ldg(tt.fix + f);  // (tile, first slot, slot count, 0)
      if (fx.x < t0 || fx.x >= t1 || fx.y < 0 || fx.z < 1 || (fx.y + fx.z) * LM1 > tt.scratch_slots) {
        bad = true;
        continue;
      }
      const int rowc = tt.tile_row[int64_t(fx.x) * R + row];
      const bool in = rowc >= 0 && rowc + LM1 <= nc;
      double acc[LM1][2];
#pragma unroll
      for (int M = 0; M < LM1; ++M) {
        const double2 v0 = in ? sG[(rowc + M) * NA + a] : make_double2(0.0, 0.0);
        acc[M][0] = v0.x;
        acc[M][1] = v0.y;
        for (int sl = fx.y; sl < fx.y + fx.z; ++sl) {
          const double2 v = scratch[sl * SLOT + (row * LM1 + M) * NA + a];
          acc[M][0] += v.x;
          acc[M][1] += v.y;
        }
      }
      finish(fx.x, acc);
    }
  }
}

// Largest intermediate L + 1 the tiled kernel is instantiated for (l_max 4).
constexpr int kTiledMaxLM1 = 9;

// Symmetric adjoint with tiled step 2 (see y3b_ace_recoupled_energy_grad_tiled):
// a CTA holds NA = 32 / rows atoms, taken from atom_order when given; steps 1
// and 3 and the mirror are those of recoupled_sym_energy_grad_kernel.  Energies
// are summed per atom over the lanes of that atom in a fixed order.
template <int NA, int TH>
__global__ void __launch_bounds__(TH, 1)
recoupled_sym_tiled_grad_kernel(SymTabs t, TileTabs tt, const double2* __restrict__ A, int64_t atom_count,
                                const int32_t* __restrict__ order, const int32_t* __restrict__ species,
                                int64_t species_count, double* __restrict__ energy, double2* __restrict__ G,
                                int32_t* status) {
  Y3B_DYNAMIC_SMEM(double2, rec_smem);
  __shared__ double red[TH / 32][NA];
  const int W = t.row_width;
  const int maxc = t.max_pass_components;
  const int cw = maxc > W ? maxc : W;
  double2* sA = rec_smem;
  double2* sGA = sA + W * NA;
  double2* sI = sGA + W * NA;
  double2* sG = sI + cw * NA;
  const int tid = threadIdx.x;
  const int lane = tid & 31, a_lane = lane % NA;
  // this warp's staging ring for step 2, after the component regions, and the
  // CTA's scratch for the partial sums of cut tiles after the rings
  unsigned char* ring = reinterpret_cast<unsigned char*>(sG + cw * NA) + (tid >> 5) * kTileStages * kStageBytes;
  double2* scratch =
      reinterpret_cast<double2*>(reinterpret_cast<unsigned char*>(sG + cw * NA) + (TH / 32) * kTileStages * kStageBytes);
  const int64_t groups = (atom_count + NA - 1) / NA;
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t first = grp * NA;
    const int nv = int(atom_count - first < NA ? atom_count - first : NA);
    int64_t idx[NA];  // the CTA's atoms (a partial group repeats its first atom, never written)
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      int64_t v = first + (a < nv ? a : 0);
      if (order != nullptr) {
        const int64_t o = order[v];
        if (o < 0 || o >= atom_count) {
          if (tid == 0 && status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
        } else {
          v = o;
        }
      }
      idx[a] = v;
    }
    // the CTA's species and weights; the staging rings hold one species'
    // weights, used when all the CTA's atoms share it (species-sorted groups)
    int za[NA];
    const double* kw[NA];
    bool uniform_z = true;
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      za[a] = species[idx[a]];
      if (za[a] < 0 || za[a] >= species_count) {
        if (tid == 0 && status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
        za[a] = 0;
      }
      kw[a] = tt.kval + int64_t(za[a]) * int64_t(tt.rows) * tt.step_count;
      uniform_z = uniform_z && za[a] == za[0];
    }
    for (int i = tid; i < W * NA; i += TH) {
      const int a = i % NA, e = i / NA;
      sA[i] = a < nv ? A[idx[a] * W + e] : make_double2(0.0, 0.0);
      sGA[i] = make_double2(0.0, 0.0);
    }
    double ep = 0.0;
    bool bad = false;
    __syncthreads();
    for (int L = 0; L < t.pass_count; ++L) {
      const int c0 = t.pass_begin[L];
      const int nc = t.pass_begin[L + 1] - c0;
      if (c0 < 0 || nc < 0 || nc > maxc || int64_t(c0) + nc > t.component_count || L >= kTiledMaxLM1) {
        bad = true;  // uniform over the block
        continue;
      }
      build_components_lanes<NA, TH>(t, sA, sI, c0, nc, W, bad);
      __syncthreads();
      switch (L) {
        case 0: tiled_adjoint_pass<1, NA, TH>(t, tt, L, c0, nc, sI, sG, kw, za, uniform_z, ring, scratch, ep, bad); break;
        case 1: tiled_adjoint_pass<2, NA, TH>(t, tt, L, c0, nc, sI, sG, kw, za, uniform_z, ring, scratch, ep, bad); break;
        case 2: tiled_adjoint_pass<3, NA, TH>(t, tt, L, c0, nc, sI, sG, kw, za, uniform_z, ring, scratch, ep, bad); break;
        case 3: tiled_adjoint_pass<4, NA, TH>(t, tt, L, c0, nc, sI, sG, kw, za, uniform_z, ring, scratch, ep, bad); break;
        case 4: tiled_adjoint_pass<5, NA, TH>(t, tt, L, c0, nc, sI, sG, kw, za, uniform_z, ring, scratch, ep, bad); break;
        case 5: tiled_adjoint_pass<6, NA, TH>(t, tt, L, c0, nc, sI, sG, kw, za, uniform_z, ring, scratch, ep, bad); break;
        case 6: tiled_adjoint_pass<7, NA, TH>(t, tt, L, c0, nc, sI, sG, kw, za, uniform_z, ring, scratch, ep, bad); break;
        case 7: tiled_adjoint_pass<8, NA, TH>(t, tt, L, c0, nc, sI, sG, kw, za, uniform_z, ring, scratch, ep, bad); break;
        default: tiled_adjoint_pass<9, NA, TH>(t, tt, L, c0, nc, sI, sG, kw, za, uniform_z, ring, scratch, ep, bad); break;
      }
      __syncthreads();
      // 3. back-propagation: lanes (work item, atom) sum their item's chunk of an
      //    A-row entry's list into a part (the component buffer is free now); each
      //    entry then adds its parts in the order t_item lists them
      {
        constexpr int R = 32 / NA;
        constexpr int NW = TH / 32;
        const int warp = tid >> 5;
        const int i0 = tt.bp_item_begin[L], i1 = tt.bp_item_begin[L + 1];
        const int ni = i1 - i0;
        const int g0 = tt.bp_group_begin[L], g1 = tt.bp_group_begin[L + 1];
        double2* part = sI;  // [ni][NA]
        if (i0 < 0 || ni < 0 || ni > cw || int64_t(i1) > tt.item_count || g0 < 0 || g1 < g0 ||
            int64_t(g1) > tt.group_count || int64_t(g1 - g0) * R < ni) {
          bad = true;  // uniform over the block
        } else {
          for (int g = g0 + warp; g < g1; g += NW) {
            const int e0 = tt.bp_group_off[g], e1 = tt.bp_group_off[g + 1];
            const int j = lane / NA;
            const int it = (g - g0) * R + j;
            if (e0 < 0 || e1 < e0 || int64_t(e1) > tt.pack_count || ((e1 - e0) % R)) {
              bad = true;  // uniform over the warp
              continue;
            }
            double2 ga = make_double2(0.0, 0.0);
            for (int e = e0 + j; e < e1; e += 8 * R) {  // eight records in flight per lane
              int4 recs[8];
#pragma unroll
              for (int u = 0; u < 8; ++u)
                recs[u] = e + u * R < e1 ? __ldg(tt.bp_pack + e + u * R) : make_int4(0, -1, 0, 0);
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const int4 rec = recs[u];  // (code, other, value lo, value hi)
                const int gi = rec.x >> 1;
                const int o = rec.y;
                if (rec.x < 0 || gi >= nc || o >= W) {
                  bad = true;
                  continue;
                }
                const double cv = __hiloint2double(rec.w, rec.z);
                double2 gg = sG[gi * NA + a_lane];
                if (rec.x & 1) gg.y = -gg.y;
                const double2 term = o < 0 ? gg : rmul(gg, sA[o * NA + a_lane]);
                ga.x = fma(cv, term.x, ga.x);
                ga.y = fma(cv, term.y, ga.y);
              }
            }
            if (it < ni) part[it * NA + a_lane] = ga;
          }
        }
        __syncthreads();
        if (!(i0 < 0 || ni < 0 || ni > cw || int64_t(i1) > tt.item_count || g0 < 0 || g1 < g0 ||
              int64_t(g1) > tt.group_count || int64_t(g1 - g0) * R < ni)) {
          for (int u = tid; u < W * NA; u += TH) {
            const int i = u / NA, a = u % NA;
            const int64_t at = int64_t(L) * W + i;
            const int j0 = tt.t_item_begin[at], j1 = tt.t_item_begin[at + 1];
            double2 acc = sGA[u];
            for (int j = j0; j < j1; ++j) {
              const int it = tt.t_item[j];
              if (it < 0 || it >= ni) {
                bad = true;
                continue;
              }
              const double2 v = part[it * NA + a];
              acc.x += v.x;
              acc.y += v.y;
            }
            sGA[u] = acc;
          }
        }
        __syncthreads();
      }
    }
    for (int u = tid; u < W * NA; u += TH) {
      const int i = u / NA, a = u % NA;
      const int mi = __ldg(t.mirror + i);
      if (mi < 0) continue;
      const int src = mi >> 1;
      if (src >= W) {
        bad = true;
        continue;
      }
      const double2 v = sGA[src * NA + a];
      const double sg = (mi & 1) ? -1.0 : 1.0;
      sGA[u] = make_double2(sg * v.x, -sg * v.y);
    }
    // per-atom energy: lanes of one atom are NA apart; shuffle down to lanes
    // 0..NA-1, then the warps in order
    for (int o = 16; o >= NA; o >>= 1) ep += __shfl_xor_sync(0xffffffffu, ep, o);
    if (lane < NA) red[tid >> 5][lane] = ep;
    __syncthreads();
    if (bad && status) atomicOr(status, Y3B_STATUS_TABLE);
    for (int i = tid; i < W * NA; i += TH) {
      const int a = i % NA, e = i / NA;
      if (a < nv) G[idx[a] * W + e] = sGA[i];
    }
    if (tid < nv) {
      double total = 0.0;
      for (int w = 0; w < TH / 32; ++w) total += red[w][tid];
      energy[idx[tid]] = total;
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace y3b
