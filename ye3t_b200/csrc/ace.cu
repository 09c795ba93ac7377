// Fused ACE evaluation: A-basis density (kernel 1) and multi-word factorized
// schedule bundle (kernel 2).
#include "edge_math.cuh"
#include "neighbors.cuh"
#include "ace_common.cuh"

namespace y3b {

constexpr int kMaxNmax = 16;

// Radial table size the density kernels are instantiated for: the smallest
// of 8, 12, 16 that holds nmax, so that the radial values stay in registers
// (the runtime nmax <= NMAXT selects the outputs).
inline int radial_table_size(int64_t nmax) { return nmax <= 8 ? 8 : (nmax <= 12 ? 12 : 16); }

// ---------------------------------------------------------------------------
// Kernel 1: A-basis density.  One warp per centre atom, DensityWarps warps per
// CTA.  Pass 1: lanes over up to 32 edges of the row compute p[z_j] R_n(r)
// (n = 1..NMAXT) and the real harmonics Y_k(r_hat) into warp-private shared
// memory.  Pass 2: lane (k, g) owns one real harmonic k and the radial channels
// n = g, g + G, ... (G = 32 / W lane groups): per edge it reads its harmonic
// once and its radial values, and accumulates in CSR order.  The complex
// Condon-Shortley harmonics are fixed combinations of two real ones
// (Yc_{l,0} = Y_{l,0}; Yc_{l,-m} = (Y_{l,m} + i Y_{l,-m}) / sqrt 2;
// Yc_{l,m} = (-1)^m (Y_{l,m} - i Y_{l,-m}) / sqrt 2), so the sums are real (half
// the multiply-adds of a complex accumulation) and lane k forms A[n, k] from its
// own sum and that of the lane of the mirrored harmonic (one shuffle per
// channel).  A is written once per atom; no atomics.
// ---------------------------------------------------------------------------
template <int LMAX, int NMAXT>
struct DensityWarps {  // up to 4 warps within 48 KB of static shared memory
  static constexpr int kPerWarp = 32 * ((NMAXT + 1) * 8 + ((LMAX + 1) * (LMAX + 1) + 1) * 8);
  static constexpr int value = 4 * kPerWarp <= 48 * 1024 ? 4 : (2 * kPerWarp <= 48 * 1024 ? 2 : 1);
};

// CTAs per SM the register allocation aims at: 6 (at most 85 registers) for the small
// instances, where it measured 16 % faster than the unbounded allocation (4 CTAs per SM);
// the larger radial tables and l_max 4 keep their registers
template <int LMAX, int NMAXT>
struct DensityMinBlocks {
  static constexpr int value = (LMAX <= 3 && NMAXT <= 8) ? 6 : 1;
};

template <int LMAX, int NMAXT>
__global__ void __launch_bounds__(32 * DensityWarps<LMAX, NMAXT>::value, DensityMinBlocks<LMAX, NMAXT>::value)
    ace_density_kernel(
    const double* __restrict__ pos, const int32_t* __restrict__ species, int64_t N,
    int64_t center_begin, int64_t count, double box, const int64_t* __restrict__ row_off,
    const int32_t* __restrict__ nbr, const double* __restrict__ pref, int64_t S, int nmax,
    double rc, double lam, ShNorm nrm, double2* __restrict__ A, int32_t* status) {
  constexpr int W = (LMAX + 1) * (LMAX + 1);
  constexpr int G = W <= 16 ? 32 / W : 1;                 // lane groups over the radial channels
  constexpr int NPL = (NMAXT + G - 1) / G;                // radial channels per lane
  constexpr int kDensityWarps = DensityWarps<LMAX, NMAXT>::value;
  __shared__ double s_rad[kDensityWarps][32][NMAXT + 1];  // +1: conflict-free pass-1 stores
  __shared__ double s_y[kDensityWarps][32][W + 1];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int k = lane % W, grp = lane / W;
  const bool owner = lane < G * W;
  // the lane's harmonic (l, m) and the lane holding the mirrored real harmonic (l, -m)
  int l = 0;
  while ((l + 1) * (l + 1) <= k) ++l;
  const int cc = l * l + l, m = k - cc;
  const int partner = lane - k + (cc - m);
  const double inv2 = 0.70710678118654752440084436210484903;
  const double sgn = (m > 0 && (m & 1)) ? -1.0 : 1.0;
  const int nout = nmax * W;
  const int64_t row0 = row_off[0];
  const int64_t warp = blockIdx.x * int64_t(kDensityWarps) + wib;
  const int64_t nwarps = int64_t(gridDim.x) * kDensityWarps;
  for (int64_t a = warp; a < count; a += nwarps) {
    const int64_t i = center_begin + a;
    const int64_t b = row_off[a] - row0, e = row_off[a + 1] - row0;
    double acc[NPL];
#pragma unroll
    for (int t = 0; t < NPL; ++t) acc[t] = 0.0;
    for (int64_t c0 = b; c0 < e; c0 += 32) {
      const int nedge = (e - c0) < 32 ? int(e - c0) : 32;
      if (lane < nedge) {
        const int64_t j = nbr[c0 + lane];
        double rv[NMAXT + 1];
        double v[W];
        double p = 0.0;
        if (j < 0 || j >= N) {
          if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
#pragma unroll
          for (int t = 0; t <= NMAXT; ++t) rv[t] = 0.0;
#pragma unroll
          for (int t = 0; t < W; ++t) v[t] = 0.0;
        } else {
          double d[3];
          min_image(pos, i, j, box, d);
          const double r = sqrt(dist2(d));
          const int zj = species[j];
          p = (zj >= 0 && zj < S) ? pref[zj] : 0.0;
          radial_basis<double>(r, rc, lam, NMAXT, rv, nullptr);
          const double sr = r > 1e-12 ? r : 1e-12;
          real_sh_unit<double, LMAX>(d[0] / sr, d[1] / sr, d[2] / sr, nrm, v, nullptr);
        }
#pragma unroll
        for (int n = 0; n < NMAXT; ++n) s_rad[wib][lane][n] = p * rv[n + 1];
#pragma unroll
        for (int t = 0; t < W; ++t) s_y[wib][lane][t] = v[t];
      }
      __syncwarp();
      if (owner) {
        for (int q = 0; q < nedge; ++q) {
          const double y = s_y[wib][q][k];
#pragma unroll
          for (int t = 0; t < NPL; ++t) {
            const int n = grp + G * t;
            if (n < NMAXT) acc[t] = fma(s_rad[wib][q][n], y, acc[t]);
          }
        }
      }
      __syncwarp();
    }
    double2* Ai = A + a * int64_t(nout);
#pragma unroll
    for (int t = 0; t < NPL; ++t) {
      const double other = __shfl_sync(0xffffffffu, acc[t], partner < 32 ? partner : lane);
      const int n = grp + G * t;
      if (owner && n < nmax) {
        double2 out;
        if (m == 0) {
          out = make_double2(acc[t], 0.0);
        } else if (m < 0) {  // (Y_{l,|m|} + i Y_{l,-|m|}) / sqrt 2
          out = make_double2(inv2 * other, inv2 * acc[t]);
        } else {             // (-1)^m (Y_{l,m} - i Y_{l,-m}) / sqrt 2
          out = make_double2(sgn * (inv2 * acc[t]), -sgn * (inv2 * other));
        }
        Ai[n * W + k] = out;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Kernel 2: the B-basis of every word, from shared memory.
//
// A CTA owns 32 atoms (lane = atom).  Its shared memory holds, per entry, one
// complex value for each of the 32 atoms ([entry][lane]: a warp reads an
// entry as one conflict-free 512-byte row):
//   * the A channels of all radial channels (entries 0 .. nmax W - 1);
//   * two slots, each holding every symmetric block Sym^k(A[n, l]) -> V_Lambda
//     of one radial channel n (symmetric_power_product_plan_contraction,
//     ye3t/runtime/symmetric_power.py:879), recomputed here when a phase
//     changes the slot's channel.
// Words are grouped in phases by the radial channels of their symmetric
// blocks (at most two per word).  Inside a phase the CTA's warps share the
// items round robin.  An item is one pass (<= 2 components) over one group
// of a word: components whose labels bind the same blocks and share M.  Its
// coefficients form a dense table over the magnetic indices of blocks
// 0..B-2; the last block's index follows from M conservation,
//   i_last = K - sum_{b < B-1} i_b,  K = M + sum_b L_b,
// and the sum is evaluated in nested order
//   B_c = sum_{i0} v0 ( sum_j C[i0, j, c] vs[j] v_last )                (B = 3)
//   B_c = sum_S sum_{i0 + i1 = S} v0 v1 ( sum_j C[i0, i1, j, c] q_j ),
//         q_j = vs[j] v_last[K - S - j]                                 (B = 4)
// with block B-2 (vs) unrolled at compile time and held in registers.
// MODE 0 writes features [N, F]; MODE 1 reduces to per-atom energy.
// ---------------------------------------------------------------------------
constexpr int kLanes = 32;  // atoms per B-basis CTA (one per lane)
constexpr int kEvalWarps = 16;
constexpr int kPadEntries = 16;  // zero entries before and after the block entries

// B = 1: a single tuple, i_0 = K.
template <typename R, int NC>
__device__ __forceinline__ void eval_b1(const Cx2<R>* __restrict__ P, const Item& it,
                                        const double* __restrict__ coef, Cx2<R>& a0, Cx2<R>& a1) {
  using C2 = typename Cplx<R>::type;
  const C2 v = P[(it.b0 + it.K) * kLanes];
  cmac(a0, __ldg(coef + it.coef), v);
  if (NC == 2) cmac(a1, __ldg(coef + it.coef + 1), v);
}

// T_c += C[j, c] * (vs[j] * v_last[kS - j]) for every j < DS.  Pk points at
// v_last[kS], so each j reads at a compile-time offset from it.  Slots whose
// last index falls outside the block have an exact-zero coefficient in the
// dense row and read a finite neighbouring entry (or the zero padding around
// the shared-memory array), so they add exactly zero and need no branch.
// Odd and even j accumulate separately (two independent FMA chains).
template <typename R, int DS, int NC>
__device__ __forceinline__ void row_sum(const Cx2<R>* __restrict__ Pk, const Cx2<R> (&vs)[DS],
                                        const double* __restrict__ crow, Cx2<R>& t0, Cx2<R>& t1) {
  using C2 = typename Cplx<R>::type;
  const CoefPair* cr2 = reinterpret_cast<const CoefPair*>(crow);
  C2 o0 = cz<C2>(), o1 = o0;
  CoefPair cc = make_double2(0.0, 0.0);
#pragma unroll
  for (int j = 0; j < DS; ++j) {
    R c0, c1 = R(0);
    if (NC == 2) {
      cc = __ldg(cr2 + j);
      c0 = R(cc.x);
      c1 = R(cc.y);
    } else {
      if ((j & 1) == 0) cc = __ldg(cr2 + (j >> 1));
      c0 = R((j & 1) ? cc.y : cc.x);
    }
    const C2 q = mul(vs[j], Pk[-j * kLanes]);
    if (j & 1) {
      cmac(o0, c0, q);
      if (NC == 2) cmac(o1, c1, q);
    } else {
      cmac(t0, c0, q);
      if (NC == 2) cmac(t1, c1, q);
    }
  }
  t0 = add(t0, o0);
  if (NC == 2) t1 = add(t1, o1);
}

template <typename R, int B, int DS, int NC>
__device__ __forceinline__ void eval_item(const Cx2<R>* __restrict__ P, const Item& it,
                                          const double* __restrict__ coef, Cx2<R>& a0, Cx2<R>& a1) {
  using C2 = typename Cplx<R>::type;
  constexpr int RW = RowWidth<DS, NC>::value;
  const int bs = B == 2 ? it.b0 : (B == 3 ? it.b1 : it.b2);  // block held in registers
  const int bl = B == 2 ? it.b1 : (B == 3 ? it.b2 : it.b3);  // last block
  C2 vs[DS];
#pragma unroll
  for (int j = 0; j < DS; ++j) vs[j] = P[(bs + j) * kLanes];
  const C2* Pl = P + bl * kLanes;
  const double* c = coef + it.coef;
  const int dl = it.dl;
  // a prefix with index sum S has tuples only for S in [smin, smax]
  const int smin = it.K - (DS - 1) - (dl - 1), smax = it.K;
  if (B == 2) {
    row_sum<R, DS, NC>(Pl + it.K * kLanes, vs, c, a0, a1);
  } else if (B == 3) {
    for (int i0 = max(0, smin); i0 < it.d0 && i0 <= smax; ++i0) {
      const int kS = it.K - i0;
      C2 t0 = cz<C2>(), t1 = t0;
      row_sum<R, DS, NC>(Pl + kS * kLanes, vs, c + i0 * RW, t0, t1);
      const C2 x0 = P[(it.b0 + i0) * kLanes];
      cfma(a0, x0, t0);
      if (NC == 2) cfma(a1, x0, t1);
    }
  } else if (DS > 7) {
    // B = 4 with a wide register block: row by row (keeps register use low)
    for (int i0 = 0; i0 < it.d0 && i0 <= smax; ++i0) {
      C2 u0 = cz<C2>(), u1 = u0;
      const int i1lo = max(0, smin - i0), i1hi = min(it.d1 - 1, smax - i0);
      for (int i1 = i1lo; i1 <= i1hi; ++i1) {
        const int kS = it.K - i0 - i1;
        C2 t0 = cz<C2>(), t1 = t0;
        row_sum<R, DS, NC>(Pl + kS * kLanes, vs, c + (i0 * it.d1 + i1) * RW, t0, t1);
        const C2 x1 = P[(it.b1 + i1) * kLanes];
        cfma(u0, x1, t0);
        if (NC == 2) cfma(u1, x1, t1);
      }
      const C2 x0 = P[(it.b0 + i0) * kLanes];
      cfma(a0, x0, u0);
      if (NC == 2) cfma(a1, x0, u1);
    }
  } else {
    // B = 4: prefixes (i0, i1) with the same index sum S read the same last-
    // block window, so loop over S: form q_j = vs[j] v_last[K - S - j] once,
    // then every prefix on the anti-diagonal only contracts its coefficient
    // row with q:  B_c += v0[i0] v1[i1] sum_j C[i0, i1, j, c] q_j.
    constexpr int DQ = DS <= 7 ? DS : 1;  // (this branch only runs for DS <= 7)
    const int s_lo = max(0, smin), s_hi = min(it.d0 - 1 + it.d1 - 1, smax);
    for (int S = s_lo; S <= s_hi; ++S) {
      const C2* Pk = Pl + (it.K - S) * kLanes;
      C2 q[DQ];
#pragma unroll
      for (int j = 0; j < DQ; ++j) q[j] = mul(vs[j], Pk[-j * kLanes]);
      const int i0lo = max(0, S - (it.d1 - 1)), i0hi = min(it.d0 - 1, S);
      for (int i0 = i0lo; i0 <= i0hi; ++i0) {
        const int i1 = S - i0;
        const CoefPair* cr2 = reinterpret_cast<const CoefPair*>(c + (i0 * it.d1 + i1) * RW);
        C2 t0 = cz<C2>(), t1 = t0, o0 = t0, o1 = t0;
        CoefPair cc = make_double2(0.0, 0.0);
#pragma unroll
        for (int j = 0; j < DQ; ++j) {
          R c0, c1 = R(0);
          if (NC == 2) {
            cc = __ldg(cr2 + j);
            c0 = R(cc.x);
            c1 = R(cc.y);
          } else {
            if ((j & 1) == 0) cc = __ldg(cr2 + (j >> 1));
            c0 = R((j & 1) ? cc.y : cc.x);
          }
          if (j & 1) {
            cmac(o0, c0, q[j]);
            if (NC == 2) cmac(o1, c1, q[j]);
          } else {
            cmac(t0, c0, q[j]);
            if (NC == 2) cmac(t1, c1, q[j]);
          }
        }
        const C2 x01 = mul(P[(it.b0 + i0) * kLanes], P[(it.b1 + i1) * kLanes]);
        cfma(a0, x01, add(t0, o0));
        if (NC == 2) cfma(a1, x01, add(t1, o1));
      }
    }
  }
}

template <typename R>
__device__ __forceinline__ void eval_dispatch(const Cx2<R>* __restrict__ P, const Item& it,
                                              const double* __restrict__ coef, Cx2<R>& a0, Cx2<R>& a1) {
  using C2 = typename Cplx<R>::type;
#define Y3B_ITEM_CASE(B, DS, NC)                                          \
  case ((B - 1) * 7 + (DS - 1) / 2) * 2 + (NC - 1):                      \
    eval_item<R, B, DS, NC>(P, it, coef, a0, a1);                           \
    break;
#define Y3B_ITEM_DS(B, DS) Y3B_ITEM_CASE(B, DS, 1) Y3B_ITEM_CASE(B, DS, 2)
#define Y3B_ITEM_B(B) \
  Y3B_ITEM_DS(B, 1) Y3B_ITEM_DS(B, 3) Y3B_ITEM_DS(B, 5) Y3B_ITEM_DS(B, 7) Y3B_ITEM_DS(B, 9) \
  Y3B_ITEM_DS(B, 11) Y3B_ITEM_DS(B, 13)
  switch (it.sel) {
    case 0: eval_b1<R, 1>(P, it, coef, a0, a1); break;
    case 1: eval_b1<R, 2>(P, it, coef, a0, a1); break;
    Y3B_ITEM_B(2)
    Y3B_ITEM_B(3)
    Y3B_ITEM_B(4)
    default: break;
  }
#undef Y3B_ITEM_B
#undef Y3B_ITEM_DS
#undef Y3B_ITEM_CASE
}

// The symmetric-output tables (outputs, term factors, term coefficients) sit
// in shared memory after the pool: a fill reads them there instead of through
// chains of L2 reads (about 5 KB for l_max 3).
struct FillTabs {
  const int4* outs;     // [so]: l^2, term begin, term end, -
  const uint32_t* fac;  // [nterm]
  const double* co;     // [nterm]
  int nterm;
};

inline size_t fill_tabs_bytes(const y3b_ace_tables& t) {
  const size_t S = size_t(t.sym_term_count);
  return size_t(16) * t.sym_output_count + ((4 * S + 15) & ~size_t(15)) + ((8 * S + 15) & ~size_t(15));
}

// All threads copy; the caller synchronises before a fill.  base is 16-byte aligned.
__device__ __forceinline__ FillTabs fill_tabs_stage(const y3b_ace_tables& t, unsigned char* base) {
  const int so = int(t.sym_output_count), S = int(t.sym_term_count);
  int4* outs = reinterpret_cast<int4*>(base);
  uint32_t* fac = reinterpret_cast<uint32_t*>(base + size_t(16) * so);
  double* co = reinterpret_cast<double*>(reinterpret_cast<unsigned char*>(fac) + ((size_t(4) * S + 15) & ~size_t(15)));
  const int4* g_outs = reinterpret_cast<const int4*>(t.sym_outputs);
  for (int i = threadIdx.x; i < so; i += blockDim.x) outs[i] = __ldg(g_outs + i);
  for (int i = threadIdx.x; i < S; i += blockDim.x) {
    fac[i] = __ldg(t.sym_term_factors + i);
    co[i] = __ldg(t.sym_term_coeff + i);
  }
  return FillTabs{outs, fac, co, S};
}

// Fill shared-memory slot `slot` with every symmetric output of radial
// channel `ch` (sym_output_tab, ace_common.cuh); a warp fills one output for
// its 32 atoms.
template <typename R, int WARPS>
__device__ __forceinline__ void fill_slot(const y3b_ace_tables& t, const FillTabs& tb, Cx2<R>* __restrict__ sm,
                                          int W, int slot, int ch, int lane, int warp) {
  const int na = int(t.nmax) * W;
  const int so = int(t.sym_output_count);
  for (int o = warp; o < so; o += WARPS) {
    const int4 r = tb.outs[o];
    sm[(na + slot * so + o) * kLanes + lane] =
        sym_output_tab(tb.fac, tb.co, r.y, min(r.z, tb.nterm), sm + (ch * W + r.x) * kLanes + lane, kLanes);
  }
}

template <typename R, int MODE, int WARPS>
__global__ void __launch_bounds__(kLanes * WARPS) ace_eval_kernel(
    y3b_ace_tables t, const Cx2<R>* __restrict__ A, int64_t N, Cx2<R>* __restrict__ feats,
    const int32_t* __restrict__ species, const double* __restrict__ weights, int64_t S,
    double* __restrict__ energy) {
  using C2 = typename Cplx<R>::type;
  extern __shared__ __align__(16) unsigned char eval_smem_raw[];
  C2* smem_all = reinterpret_cast<C2*>(eval_smem_raw);
  __shared__ double red[WARPS][kLanes];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int W = int((t.lmax + 1) * (t.lmax + 1));
  const int na = int(t.nmax) * W;
  const int64_t a = blockIdx.x * int64_t(kLanes) + lane;
  const bool live = a < N;
  // zero everything (padding and slots), then the A channels
  const int total = (int(t.smem_entries) + 2 * kPadEntries) * kLanes;
  for (int e = threadIdx.x; e < total; e += blockDim.x) smem_all[e] = cz<C2>();
  const FillTabs tb = fill_tabs_stage(t, eval_smem_raw + size_t(total) * sizeof(C2));
  __syncthreads();
  C2* sm = smem_all + kPadEntries * kLanes;
  for (int e = warp; e < na; e += WARPS)
    sm[e * kLanes + lane] = live ? A[a * na + e] : cz<C2>();
  const double* wz = weights;
  if (MODE == 1) {
    int z = live ? species[a] : 0;
    if (z < 0 || z >= S) z = 0;
    wz = weights + int64_t(z) * t.feature_count;
  }
  const C2* P = sm + lane;
  const int4* items = reinterpret_cast<const int4*>(t.items);
  const int4* phases = reinterpret_cast<const int4*>(t.phases);
  int cur0 = -2, cur1 = -2;
  double e_acc = 0.0;
  for (int ph = 0; ph < t.phase_count; ++ph) {
    const int4 pr = __ldg(phases + ph);
    if (pr.x != cur0 || pr.y != cur1) {
      __syncthreads();  // previous phase's items are done with the slots (and A is loaded)
      if (pr.x != cur0) fill_slot<R, WARPS>(t, tb, sm, W, 0, pr.x, lane, warp);
      // (the second slot exists only in pools sized for it)
      if (pr.y != cur1 && pr.y >= 0 && t.smem_entries >= na + 2 * t.sym_output_count)
        fill_slot<R, WARPS>(t, tb, sm, W, 1, pr.y, lane, warp);
      __syncthreads();
      cur0 = pr.x;
      cur1 = pr.y;
    }
    for (int i = pr.z + warp; i < pr.w; i += WARPS) {
      const Item it = load_item(items, i);
      C2 a0 = cz<C2>(), a1 = a0;
      eval_dispatch<R>(P, it, t.item_coef, a0, a1);
      if (MODE == 0) {
        if (live) {
          feats[a * t.feature_count + it.f0] = a0;
          if (it.f1 >= 0) feats[a * t.feature_count + it.f1] = a1;
        }
      } else {
        e_acc = fma(__ldg(wz + it.f0), double(a0.x), e_acc);
        if (it.f1 >= 0) e_acc = fma(__ldg(wz + it.f1), double(a1.x), e_acc);
      }
    }
  }
  if (MODE == 1) {
    red[warp][lane] = e_acc;
    __syncthreads();
    if (warp == 0 && live) {
      double s = 0.0;
      for (int w = 0; w < WARPS; ++w) s += red[w][lane];
      energy[a] = s;
    }
  }
}

inline size_t eval_smem_bytes(const y3b_ace_tables& t, size_t complex_size = sizeof(double2)) {
  return size_t(t.smem_entries + 2 * kPadEntries) * kLanes * complex_size + fill_tabs_bytes(t);
}

int check_tables(const y3b_ace_tables* t) {
  Y3B_CHECK_ARG(t != nullptr, "null tables");
  Y3B_CHECK_ARG(t->nmax >= 1 && t->nmax <= kMaxNmax, "nmax must be in [1, %d]", kMaxNmax);
  Y3B_CHECK_ARG(t->lmax >= 0 && t->lmax <= 6, "lmax must be in [0, 6]");
  Y3B_CHECK_ARG(t->item_count >= 0 && t->feature_count >= 0 && t->phase_count >= 1, "bad table sizes");
  Y3B_CHECK_ARG(t->item_count == 0 || (t->items && t->item_coef && t->phases), "null item tables");
  Y3B_CHECK_ARG(t->smem_entries >= t->nmax * (t->lmax + 1) * (t->lmax + 1) + t->sym_output_count,
                "shared-memory entry count too small");
  Y3B_CHECK_ARG(t->sym_term_count >= 0 && (t->sym_output_count == 0 || t->sym_term_count > 0),
                "symmetric term count missing");
  Y3B_CHECK_ARG(eval_smem_bytes(*t) <= 200 * 1024, "bundle needs %lld bytes of shared memory per CTA (max 200 KB)",
                (long long)eval_smem_bytes(*t));
  return Y3B_OK;
}

template <typename R, int MODE, int WARPS>
int launch_eval_w(const y3b_ace_tables* t, const void* A, int64_t n, typename Cplx<R>::type* feats,
                  const int32_t* species, const double* weights, int64_t S, double* energy, cudaStream_t s,
                  size_t smem) {
  using C2 = typename Cplx<R>::type;
  Y3B_CUDA_TRY(cudaFuncSetAttribute(ace_eval_kernel<R, MODE, WARPS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)));
  const int64_t grid = (n + kLanes - 1) / kLanes;
  Y3B_CHECK_ARG(grid < (int64_t(1) << 31), "too many atoms");
  ace_eval_kernel<R, MODE, WARPS><<<int(grid), kLanes * WARPS, smem, s>>>(*t, static_cast<const C2*>(A), n, feats,
                                                                          species, weights, S, energy);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

// Pools small enough for two CTAs per SM run 8-warp CTAs (two of them share
// an SM, so one's phase barriers overlap the other's items); larger pools run
// one 16-warp CTA per SM.
template <typename R, int MODE>
int launch_eval(const y3b_ace_tables* t, const void* A, int64_t n, typename Cplx<R>::type* feats,
                const int32_t* species, const double* weights, int64_t S, double* energy, cudaStream_t s) {
  using C2 = typename Cplx<R>::type;
  const size_t smem = eval_smem_bytes(*t, sizeof(C2));
  if (2 * (smem + 2048) <= 227 * 1024)
    return launch_eval_w<R, MODE, 8>(t, A, n, feats, species, weights, S, energy, s, smem);
  return launch_eval_w<R, MODE, kEvalWarps>(t, A, n, feats, species, weights, S, energy, s, smem);
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
#define Y3B_DENSITY_LAUNCH(L, NT)                                                                    \
  ace_density_kernel<L, NT><<<int(std::min<int64_t>((center_count + DensityWarps<L, NT>::value - 1) /      \
                                                        DensityWarps<L, NT>::value,                        \
                                                    int64_t(kSMs) * 128)),                                 \
                              32 * DensityWarps<L, NT>::value, 0, s>>>(                                    \
      positions, species, atom_count, center_begin, center_count, box, row_offsets, neighbors,            \
      species_prefactor, species_count, int(nmax), cutoff, lambda, nrm, static_cast<double2*>(A), status)
#define Y3B_DENSITY_CASE(L)                                                                            \
  case L:                                                                                              \
    if (nt == 8) Y3B_DENSITY_LAUNCH(L, 8);                                                             \
    else if (nt == 12) Y3B_DENSITY_LAUNCH(L, 12);                                                      \
    else Y3B_DENSITY_LAUNCH(L, 16);                                                                    \
    break;
  const int nt = radial_table_size(nmax);
  switch (lmax) {
    Y3B_DENSITY_CASE(0)
    Y3B_DENSITY_CASE(1)
    Y3B_DENSITY_CASE(2)
    Y3B_DENSITY_CASE(3)
    Y3B_DENSITY_CASE(4)
    default:
      return fail(Y3B_ERR_UNSUPPORTED, "ace_density: lmax %lld not built (0..4)", (long long)lmax);
  }
#undef Y3B_DENSITY_LAUNCH
#undef Y3B_DENSITY_CASE
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_ace_features(const y3b_ace_tables* tables, const void* A, int64_t atom_count,
                                void* features, void* stream) {
  if (int rc = check_tables(tables)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && features, "null pointer argument");
  return launch_eval<double, 0>(tables, A, atom_count, static_cast<double2*>(features), nullptr, nullptr, 0,
                                nullptr, as_stream(stream));
}

extern "C" int y3b_ace_features_typed(int dtype, const y3b_ace_tables* tables, const void* A, int64_t atom_count,
                                      void* features, void* stream) {
  if (int rc = check_tables(tables)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && features, "null pointer argument");
  if (dtype == Y3B_C128)
    return launch_eval<double, 0>(tables, A, atom_count, static_cast<double2*>(features), nullptr, nullptr, 0,
                                  nullptr, as_stream(stream));
  if (dtype == Y3B_C64)
    return launch_eval<float, 0>(tables, A, atom_count, static_cast<float2*>(features), nullptr, nullptr, 0,
                                 nullptr, as_stream(stream));
  return fail(Y3B_ERR_ARGUMENT, "ace_features: dtype must be C64 or C128 (got %d)", dtype);
}

extern "C" int y3b_ace_energy(const y3b_ace_tables* tables, const void* A, int64_t atom_count,
                              const int32_t* species, const double* weights, int64_t species_count,
                              double* energy, void* stream) {
  if (int rc = check_tables(tables)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && species && weights && energy && species_count > 0, "null pointer argument");
  return launch_eval<double, 1>(tables, A, atom_count, nullptr, species, weights, species_count, energy,
                                as_stream(stream));
}
