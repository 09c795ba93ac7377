// Force path of the fused ACE evaluation (the reverse of kernels 1 and 2).
//
// E = sum_i sum_f w[z_i, f] Re(B_if).  B is a polynomial (holomorphic) in the
// A-basis, so dE = Re(sum G dA) with G = sum_f w_f dB_f/dA; the reference
// obtains the same quantity by torch autograd through its schedule
// evaluator, symmetric-power adjoint (execution_plan_cuda.cu:5272) and
// density_accumulate_adjoint (execution_plan.py:7987).
//
//  1. ace_grad_kernel: per atom, E_i and G_i = dE_i/dA_i (B-basis adjoint).
//  2. ace_edge_grad_kernel: per edge e = (i -> j), g_e = dE_i/dd_e with
//     d_e = r_j - r_i, from G_i and the radial / harmonic derivatives
//     (plain_site_basis_product_adjoint, execution_plan.py:7790, fused).
//  3. forces: F_k = sum_{e in row k} (g_e - g_rev(e)) (deterministic gather over
//     the symmetric neighbour list), or a scatter into a partial force array
//     when only some rows are local (atom-block partition).
#include "ace_common.cuh"
#include "edge_math.cuh"
#include "neighbors.cuh"

namespace y3b {

namespace {

// A CTA holds values and gradient accumulators of 16 atoms in shared memory
// ([entry][atom]); lanes l and l + 16 of a warp work on atom l and split each
// item's outer iterations between them.
constexpr int kGA = 16;
constexpr int kGWarps = 8;
constexpr int kGPad = 16;  // zero entries before and after the block entries

struct Tile {
  const double2* V;  // V[e * kGA]: value of entry e for this lane's atom
  double2* G;        // G[e * kGA]: its gradient accumulator
};

__device__ __forceinline__ double2 vat(const Tile& tl, int e) { return tl.V[e * kGA]; }

// Gradient entries are shared by the CTA's warps, so accumulation is atomic
// (the order of these partial sums is not fixed; forces agree run to run to
// rounding).
__device__ __forceinline__ void gacc(const Tile& tl, int e, double2 v) {
  atomicAdd(&tl.G[e * kGA].x, v.x);
  atomicAdd(&tl.G[e * kGA].y, v.y);
}

__device__ __forceinline__ double2 cscale(double c, double2 v) { return make_double2(c * v.x, c * v.y); }

__device__ __forceinline__ double2 shfl_half(double2 v) {
  return make_double2(__shfl_xor_sync(0xffffffffu, v.x, 16), __shfl_xor_sync(0xffffffffu, v.y, 16));
}

// Readout-weighted coefficient j of a row: w0 C[j, 0] + w1 C[j, 1].
template <int NC>
__device__ __forceinline__ double wcoef(const double* __restrict__ crow, int j, double w0, double w1) {
  if (NC == 2) {
    const double2 c = __ldg(reinterpret_cast<const double2*>(crow) + j);
    return w0 * c.x + w1 * c.y;
  }
  return w0 * __ldg(crow + j);
}

// Register window over the last block's gradient: a[t] belongs to index
// base - t.  A half-warp's bases fall by 2 per outer step, so each step
// flushes the two entries that no later step can reach and shifts by two.
template <int DS>
__device__ __forceinline__ void win_step2(const Tile& tl, int bl, int dl, int base, double2 (&a)[DS]) {
#pragma unroll
  for (int t = 0; t < 2 && t < DS; ++t) {
    const int li = base - t;
    if (li >= 0 && li < dl && (a[t].x != 0.0 || a[t].y != 0.0)) gacc(tl, bl + li, a[t]);
  }
#pragma unroll
  for (int t = 0; t < DS; ++t) a[t] = t + 2 < DS ? a[t + 2] : make_double2(0.0, 0.0);
}

template <int DS>
__device__ __forceinline__ void win_flush(const Tile& tl, int bl, int dl, int base, const double2 (&a)[DS]) {
#pragma unroll
  for (int t = 0; t < DS; ++t) {
    const int li = base - t;
    if (li >= 0 && li < dl && (a[t].x != 0.0 || a[t].y != 0.0)) gacc(tl, bl + li, a[t]);
  }
}

// Half-warp partial sums of register gradients are combined, then flushed once.
template <int D>
__device__ __forceinline__ void flush_pair(const Tile& tl, int base, int count, double2 (&g)[D], int half) {
#pragma unroll
  for (int j = 0; j < D; ++j) {
    const double2 s = add(g[j], shfl_half(g[j]));
    if (half == 0 && j < count && (s.x != 0.0 || s.y != 0.0)) gacc(tl, base + j, s);
  }
}

template <int NC>
__device__ __forceinline__ void adj_b1(const Tile& tl, const Item& it, const double* __restrict__ coef, double w0,
                                       double w1, int half, double& e) {
  if (half) return;
  const double c = w0 * __ldg(coef + it.coef) + (NC == 2 ? w1 * __ldg(coef + it.coef + 1) : 0.0);
  const double2 v = vat(tl, it.b0 + it.K);
  e += c * v.x;
  gacc(tl, it.b0 + it.K, make_double2(c, 0.0));
}

// One row with prefix value x:  F += x sum_j c_j vs_j vl[kS - j].  Returns
// T = sum_j c_j vs_j vl_j; adds x c_j vl_j to gvs[j] and x c_j vs_j to the
// last block's window (win[j] belongs to index kS - j).
template <int DS, int NC>
__device__ __forceinline__ double2 adj_row(const Tile& tl, int bl, int kS, int dl, const double2 (&vs)[DS],
                                           double2 (&gvs)[DS], double2 (&win)[DS], const double* __restrict__ crow,
                                           double w0, double w1, double2 x) {
  double2 T = make_double2(0.0, 0.0);
#pragma unroll
  for (int j = 0; j < DS; ++j) {
    const int li = kS - j;
    if (li >= 0 && li < dl) {
      const double c = wcoef<NC>(crow, j, w0, w1);
      const double2 vl = vat(tl, bl + li);
      cmac(T, c, mul(vs[j], vl));
      const double2 xc = cscale(c, x);
      cfma(gvs[j], xc, vl);
      cfma(win[j], xc, vs[j]);
    }
  }
  return T;
}

template <int B, int DS, int NC>
__device__ __forceinline__ void adj_item(const Tile& tl, const Item& it, const double* __restrict__ coef,
                                         double w0, double w1, int half, double& e) {
  constexpr int RW = RowWidth<DS, NC>::value;
  const int bs = B == 2 ? it.b0 : (B == 3 ? it.b1 : it.b2);
  const int bl = B == 2 ? it.b1 : (B == 3 ? it.b2 : it.b3);
  double2 vs[DS], gvs[DS], win[DS];
#pragma unroll
  for (int j = 0; j < DS; ++j) {
    vs[j] = vat(tl, bs + j);
    gvs[j] = make_double2(0.0, 0.0);
    win[j] = make_double2(0.0, 0.0);
  }
  const double* c = coef + it.coef;
  const int dl = it.dl;
  const int smin = it.K - (DS - 1) - (dl - 1), smax = it.K;
  if (B == 2) {
    if (half == 0) {
      const double2 T = adj_row<DS, NC>(tl, bl, it.K, dl, vs, gvs, win, c, w0, w1, make_double2(1.0, 0.0));
      e += T.x;
      win_flush<DS>(tl, bl, dl, it.K, win);
    }
  } else if (B == 3) {
    int i0 = max(0, smin) + half;
    for (; i0 < it.d0 && i0 <= smax; i0 += 2) {
      const double2 x0 = vat(tl, it.b0 + i0);
      const double2 T = adj_row<DS, NC>(tl, bl, it.K - i0, dl, vs, gvs, win, c + i0 * RW, w0, w1, x0);
      e += x0.x * T.x - x0.y * T.y;
      gacc(tl, it.b0 + i0, T);
      win_step2<DS>(tl, bl, dl, it.K - i0, win);
    }
    win_flush<DS>(tl, bl, dl, it.K - i0, win);
  } else if (DS > 7) {
    // 4 blocks with a wide register block: rows in (i0, i1) order, last-block
    // gradients added directly
    for (int i0 = half; i0 < it.d0 && i0 <= smax; i0 += 2) {
      const double2 x0 = vat(tl, it.b0 + i0);
      double2 gx0 = make_double2(0.0, 0.0);
      const int i1lo = max(0, smin - i0), i1hi = min(it.d1 - 1, smax - i0);
      for (int i1 = i1lo; i1 <= i1hi; ++i1) {
        const double2 x1 = vat(tl, it.b1 + i1);
        const double2 x01 = mul(x0, x1);
        const int kS = it.K - i0 - i1;
#pragma unroll
        for (int j = 0; j < DS; ++j) win[j] = make_double2(0.0, 0.0);
        const double2 T = adj_row<DS, NC>(tl, bl, kS, dl, vs, gvs, win, c + (i0 * it.d1 + i1) * RW, w0, w1, x01);
        win_flush<DS>(tl, bl, dl, kS, win);
        e += x01.x * T.x - x01.y * T.y;
        cfma(gx0, x1, T);
        gacc(tl, it.b1 + i1, mul(x0, T));
      }
      gacc(tl, it.b0 + i0, gx0);
    }
  } else {
    // 4 blocks, register block <= 7: anti-diagonals S = i0 + i1 share
    // q_j = vs_j vl[K - S - j].  Both half-warps take the same S and split its
    // rows (alternate i0); R_j = sum_rows x0 x1 C[.., j] is combined across
    // the halves, and half 0 adds the register-block and last-block
    // gradients (the last block through a window that slides by one per S).
    constexpr int DQ = DS <= 7 ? DS : 1;
    double2 wq[DQ];
#pragma unroll
    for (int j = 0; j < DQ; ++j) wq[j] = make_double2(0.0, 0.0);
    const int s_lo = max(0, smin), s_hi = min(it.d0 - 1 + it.d1 - 1, smax);
    int S = s_lo;
    for (; S <= s_hi; ++S) {
      const int kS = it.K - S;
      double2 q[DQ], R[DQ];
#pragma unroll
      for (int j = 0; j < DQ; ++j) {
        q[j] = mul(vs[j], vat(tl, bl + kS - j));  // out-of-block slots read finite padding; their coefficients are 0
        R[j] = make_double2(0.0, 0.0);
      }
      const int i0lo = max(0, S - (it.d1 - 1)), i0hi = min(it.d0 - 1, S);
      for (int i0 = i0lo + half; i0 <= i0hi; i0 += 2) {
        const int i1 = S - i0;
        const double* crow = c + (i0 * it.d1 + i1) * RW;
        const double2 x0 = vat(tl, it.b0 + i0), x1 = vat(tl, it.b1 + i1);
        const double2 x01 = mul(x0, x1);
        double2 T = make_double2(0.0, 0.0);
#pragma unroll
        for (int j = 0; j < DQ; ++j) {
          const double cj = wcoef<NC>(crow, j, w0, w1);
          cmac(T, cj, q[j]);
          cmac(R[j], cj, x01);
        }
        e += x01.x * T.x - x01.y * T.y;
        gacc(tl, it.b0 + i0, mul(x1, T));
        gacc(tl, it.b1 + i1, mul(x0, T));
      }
#pragma unroll
      for (int j = 0; j < DQ; ++j) {
        R[j] = add(R[j], shfl_half(R[j]));
        if (half == 0) {
          cfma(gvs[j], R[j], vat(tl, bl + kS - j));
          cfma(wq[j], R[j], vs[j]);
        }
      }
      if (half == 0) {
        // entry kS is final: later diagonals reach only indices below it
        if (kS >= 0 && kS < dl && (wq[0].x != 0.0 || wq[0].y != 0.0)) gacc(tl, bl + kS, wq[0]);
#pragma unroll
        for (int j = 0; j < DQ; ++j) wq[j] = j + 1 < DQ ? wq[j + 1] : make_double2(0.0, 0.0);
      }
    }
    if (half == 0) win_flush<DQ>(tl, bl, dl, it.K - S, wq);
  }
  flush_pair<DS>(tl, bs, DS, gvs, half);
}

__device__ __forceinline__ void adj_dispatch(const Tile& tl, const Item& it, const double* __restrict__ coef,
                                             double w0, double w1, int half, double& e) {
#define Y3B_ADJ_CASE(B, DS, NC)                         \
  case ((B - 1) * 7 + (DS - 1) / 2) * 2 + (NC - 1):     \
    adj_item<B, DS, NC>(tl, it, coef, w0, w1, half, e); \
    break;
#define Y3B_ADJ_DS(B, DS) Y3B_ADJ_CASE(B, DS, 1) Y3B_ADJ_CASE(B, DS, 2)
#define Y3B_ADJ_B(B) \
  Y3B_ADJ_DS(B, 1) Y3B_ADJ_DS(B, 3) Y3B_ADJ_DS(B, 5) Y3B_ADJ_DS(B, 7) Y3B_ADJ_DS(B, 9) \
  Y3B_ADJ_DS(B, 11) Y3B_ADJ_DS(B, 13)
  switch (it.sel) {
    case 0: adj_b1<1>(tl, it, coef, w0, w1, half, e); break;
    case 1: adj_b1<2>(tl, it, coef, w0, w1, half, e); break;
    Y3B_ADJ_B(2)
    Y3B_ADJ_B(3)
    Y3B_ADJ_B(4)
    default: break;
  }
#undef Y3B_ADJ_B
#undef Y3B_ADJ_DS
#undef Y3B_ADJ_CASE
}

// Symmetric slot: fill values from A.  Threads cover (atom, output) pairs.
__device__ __forceinline__ void grad_fill_slot(const y3b_ace_tables& t, double2* __restrict__ val, int W, int slot,
                                               int ch) {
  const int na = int(t.nmax) * W, so = int(t.sym_output_count);
  const int4* outs = reinterpret_cast<const int4*>(t.sym_outputs);
  const int atom = threadIdx.x % kGA;
  for (int o = threadIdx.x / kGA; o < so; o += blockDim.x / kGA) {
    const int4 r = __ldg(outs + o);
    val[(na + slot * so + o) * kGA + atom] = sym_output(t, r.y, r.z, val + (ch * W + r.x) * kGA + atom, kGA);
  }
}

// Pull a slot's gradients back to the A entries of its radial channel:
// d/dx_c of coeff prod_k x_{f_k} is, for each distinct component c (first
// occurrence p), multiplicity(c) coeff prod_{k != p} x_{f_k}.  Clears the slot.
__device__ __forceinline__ void grad_pull_slot(const y3b_ace_tables& t, const double2* __restrict__ val,
                                               double2* __restrict__ grad, int W, int slot, int ch) {
  const int na = int(t.nmax) * W, so = int(t.sym_output_count);
  const int4* outs = reinterpret_cast<const int4*>(t.sym_outputs);
  const int atom = threadIdx.x % kGA;
  for (int o = threadIdx.x / kGA; o < so; o += blockDim.x / kGA) {
    double2* gslot = grad + (na + slot * so + o) * kGA + atom;
    const double2 g = *gslot;
    *gslot = make_double2(0.0, 0.0);
    if (g.x == 0.0 && g.y == 0.0) continue;
    const int4 r = __ldg(outs + o);
    const double2* x = val + (ch * W + r.x) * kGA + atom;
    double2* gx = grad + (ch * W + r.x) * kGA + atom;
    for (int q = r.y; q < r.z; ++q) {
      const uint32_t f = __ldg(t.sym_term_factors + q);
      const double cq = __ldg(t.sym_term_coeff + q);
      int fk[4], nf = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int ci = (f >> (8 * k)) & 255;
        if (ci != 255 && nf == k) fk[nf++] = ci;
      }
      for (int p = 0; p < nf; ++p) {
        if (p > 0 && fk[p] == fk[p - 1]) continue;
        int mult = 0;
        double2 prod = make_double2(cq, 0.0);
        for (int k = 0; k < nf; ++k) {
          if (fk[k] == fk[p]) ++mult;
          if (k != p) prod = mul(prod, x[fk[k] * kGA]);
        }
        const double2 d = mul(g, cscale(double(mult), prod));
        atomicAdd(&gx[fk[p] * kGA].x, d.x);
        atomicAdd(&gx[fk[p] * kGA].y, d.y);
      }
    }
  }
}

__global__ void __launch_bounds__(32 * kGWarps) ace_grad_kernel(y3b_ace_tables t, const double2* __restrict__ A,
                                                                int64_t N, const int32_t* __restrict__ species,
                                                                const double* __restrict__ weights, int64_t S,
                                                                double* __restrict__ energy,
                                                                double2* __restrict__ dEdA) {
  extern __shared__ double2 gsm[];
  __shared__ double red[kGWarps][kGA];
  const int W = int((t.lmax + 1) * (t.lmax + 1));
  const int na = int(t.nmax) * W;
  const int rows = int(t.smem_entries) + 2 * kGPad;
  for (int e = threadIdx.x; e < 2 * rows * kGA; e += blockDim.x) gsm[e] = make_double2(0.0, 0.0);
  __syncthreads();
  double2* val = gsm + kGPad * kGA;
  double2* grad = gsm + (rows + kGPad) * kGA;
  {
    const int la = threadIdx.x % kGA;  // loader thread's atom
    const int64_t aa = blockIdx.x * int64_t(kGA) + la;
    for (int e = threadIdx.x / kGA; e < na; e += blockDim.x / kGA)
      val[e * kGA + la] = aa < N ? A[aa * na + e] : make_double2(0.0, 0.0);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int atom = lane & (kGA - 1), half = lane >> 4;
  const int64_t a = blockIdx.x * int64_t(kGA) + atom;
  const bool live = a < N;
  int z = live ? species[a] : 0;
  if (z < 0 || z >= S) z = 0;
  const double* wz = weights + int64_t(z) * t.feature_count;
  const Tile tl{val + atom, grad + atom};
  const int4* items = reinterpret_cast<const int4*>(t.items);
  const int4* phases = reinterpret_cast<const int4*>(t.phases);
  int cur0 = -2, cur1 = -2;
  double e_acc = 0.0;
  for (int ph = 0; ph < t.phase_count; ++ph) {
    const int4 pr = __ldg(phases + ph);
    if (pr.x != cur0 || pr.y != cur1) {
      __syncthreads();  // the previous phase is done with the slots (and A is loaded)
      if (pr.x != cur0 && cur0 >= 0) grad_pull_slot(t, val, grad, W, 0, cur0);
      if (pr.y != cur1 && cur1 >= 0) grad_pull_slot(t, val, grad, W, 1, cur1);
      __syncthreads();
      if (pr.x != cur0) grad_fill_slot(t, val, W, 0, pr.x);
      if (pr.y != cur1 && pr.y >= 0) grad_fill_slot(t, val, W, 1, pr.y);
      __syncthreads();
      cur0 = pr.x;
      cur1 = pr.y;
    }
    for (int i = pr.z + warp; i < pr.w; i += kGWarps) {
      const Item it = load_item(items, i);
      const double w0 = __ldg(wz + it.f0);
      const double w1 = it.f1 >= 0 ? __ldg(wz + it.f1) : 0.0;
      adj_dispatch(tl, it, t.item_coef, w0, w1, half, e_acc);
    }
  }
  __syncthreads();
  if (cur0 >= 0) grad_pull_slot(t, val, grad, W, 0, cur0);
  if (cur1 >= 0) grad_pull_slot(t, val, grad, W, 1, cur1);
  e_acc += __shfl_xor_sync(0xffffffffu, e_acc, 16);
  if (half == 0) red[warp][atom] = e_acc;
  __syncthreads();
  if (threadIdx.x < kGA) {
    const int64_t aa = blockIdx.x * int64_t(kGA) + threadIdx.x;
    double s = 0.0;
    for (int w = 0; w < kGWarps; ++w) s += red[w][threadIdx.x];
    if (aa < N) energy[aa] = s;
  }
  {
    const int la = threadIdx.x % kGA;
    const int64_t aa = blockIdx.x * int64_t(kGA) + la;
    for (int e = threadIdx.x / kGA; e < na; e += blockDim.x / kGA)
      if (aa < N) dEdA[aa * na + e] = grad[e * kGA + la];
  }
}

// ---------------------------------------------------------------------------
// Edge gradients: one warp per centre i; lanes over its edges.  With
// A[n, lm] = sum_j p_j R_n(r) Yc_lm(d),  g_e = dE_i/dd_e =
//   p_j ( d_hat sum_n R'_n Re(sum_lm G[n,lm] Yc_lm) + sum_n R_n Re(sum_lm G[n,lm] grad Yc_lm) ).
// ---------------------------------------------------------------------------
constexpr int kEdgeWarps = 2;

template <int LMAX>
__global__ void __launch_bounds__(32 * kEdgeWarps) ace_edge_grad_kernel(
    const double* __restrict__ pos, const int32_t* __restrict__ species, int64_t N, int64_t center_begin,
    int64_t count, double box, const int64_t* __restrict__ row_off, const int32_t* __restrict__ nbr,
    const double* __restrict__ pref, int64_t S, int nmax, double rc, double lam, ShNorm nrm,
    const double2* __restrict__ dEdA, double* __restrict__ edge_grad, int32_t* status) {
  constexpr int W = (LMAX + 1) * (LMAX + 1);
  __shared__ double2 sG[kEdgeWarps][16 * W];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int na = nmax * W;
  const int64_t row0 = row_off[0];
  for (int64_t c = blockIdx.x * int64_t(kEdgeWarps) + wib; c < count; c += int64_t(gridDim.x) * kEdgeWarps) {
    const int64_t i = center_begin + c;
    for (int k = lane; k < na; k += 32) sG[wib][k] = dEdA[c * na + k];
    __syncwarp();
    const int64_t b = row_off[c] - row0, e_end = row_off[c + 1] - row0;
    for (int64_t e = b + lane; e < e_end; e += 32) {
      const int64_t j = nbr[e];
      double gx = 0.0, gy = 0.0, gz = 0.0;
      if (j < 0 || j >= N) {
        if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
      } else {
        double d[3];
        min_image(pos, i, j, box, d);
        const double r = sqrt(dist2(d));
        const int zj = species[j];
        const double p = (zj >= 0 && zj < S) ? pref[zj] : 0.0;
        double rv[17], rd[17];
        radial_basis<double>(r, rc, lam, nmax, rv, rd);
        const double eps = 1e-12;
        const double sr = r > eps ? r : eps;
        const double u[3] = {d[0] / sr, d[1] / sr, d[2] / sr};
        double v[W], g[W][3];
        real_sh_unit<double, LMAX>(u[0], u[1], u[2], nrm, v, g);
        // Cartesian gradients of the real harmonics, in place: J = (I - u u^T) / |d|
        // (I / eps below eps), as ye3t_runtime_core.cpp:819-834
#pragma unroll
        for (int k = 0; k < W; ++k) {
          const double gu = r > eps ? g[k][0] * u[0] + g[k][1] * u[1] + g[k][2] * u[2] : 0.0;
#pragma unroll
          for (int ax = 0; ax < 3; ++ax) g[k][ax] = (g[k][ax] - gu * u[ax]) / sr;
        }
        double acc_r = 0.0, acc_v[3] = {0.0, 0.0, 0.0};
        const double inv2 = 0.70710678118654752440084436210484903;
#pragma unroll
        for (int l = 0; l <= LMAX; ++l) {
          const int cidx = l * l + l;
#pragma unroll
          for (int m = -l; m <= l; ++m) {
            // complex harmonic and its gradient from the real ones
            // (Yc_{l,-m} = (R_{+m} + i R_{-m}) / sqrt2, Yc_{l,+m} = (-1)^m (R_{+m} - i R_{-m}) / sqrt2)
            double yr, yi, dr[3], di[3];
            if (m == 0) {
              yr = v[cidx];
              yi = 0.0;
#pragma unroll
              for (int ax = 0; ax < 3; ++ax) {
                dr[ax] = g[cidx][ax];
                di[ax] = 0.0;
              }
            } else if (m < 0) {
              const int pp = cidx - m, nn = cidx + m;
              yr = inv2 * v[pp];
              yi = inv2 * v[nn];
#pragma unroll
              for (int ax = 0; ax < 3; ++ax) {
                dr[ax] = inv2 * g[pp][ax];
                di[ax] = inv2 * g[nn][ax];
              }
            } else {
              const double sg = (m & 1) ? -1.0 : 1.0;
              const int pp = cidx + m, nn = cidx - m;
              yr = sg * (inv2 * v[pp]);
              yi = sg * (inv2 * -v[nn]);
#pragma unroll
              for (int ax = 0; ax < 3; ++ax) {
                dr[ax] = sg * (inv2 * g[pp][ax]);
                di[ax] = sg * (inv2 * -g[nn][ax]);
              }
            }
            const int lm = cidx + m;
            for (int n = 0; n < nmax; ++n) {
              const double2 G = sG[wib][n * W + lm];
              acc_r += rd[n + 1] * (G.x * yr - G.y * yi);
              const double Rn = rv[n + 1];
#pragma unroll
              for (int ax = 0; ax < 3; ++ax) acc_v[ax] += Rn * (G.x * dr[ax] - G.y * di[ax]);
            }
          }
        }
        gx = p * (acc_r * u[0] + acc_v[0]);
        gy = p * (acc_r * u[1] + acc_v[1]);
        gz = p * (acc_r * u[2] + acc_v[2]);
      }
      edge_grad[3 * e + 0] = gx;
      edge_grad[3 * e + 1] = gy;
      edge_grad[3 * e + 2] = gz;
    }
    __syncwarp();
  }
}

// F_k = sum_{e in row k} (g_e - g_rev(e)); rows cover every atom and are
// sorted, so rev(e) is found by binary search in row nbr[e].
__global__ void forces_gather_kernel(const int64_t* __restrict__ row_off, const int32_t* __restrict__ nbr,
                                     int64_t N, const double* __restrict__ g, double* __restrict__ F,
                                     int32_t* status) {
  for (int64_t k = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; k < N; k += int64_t(gridDim.x) * blockDim.x) {
    double f[3] = {0.0, 0.0, 0.0};
    for (int64_t e = row_off[k]; e < row_off[k + 1]; ++e) {
      const int64_t j = nbr[e];
      int64_t rev = -1;
      if (j >= 0 && j < N) {
        int64_t lo = row_off[j], hi = row_off[j + 1] - 1;
        while (lo <= hi) {
          const int64_t mid = (lo + hi) >> 1;
          const int32_t v = nbr[mid];
          if (v == k) {
            rev = mid;
            break;
          }
          if (v < k) lo = mid + 1;
          else hi = mid - 1;
        }
      }
      if (rev < 0) {
        if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
        continue;
      }
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) f[ax] += g[3 * e + ax] - g[3 * rev + ax];
    }
#pragma unroll
    for (int ax = 0; ax < 3; ++ax) F[3 * k + ax] = f[ax];
  }
}

// Partial forces of the local rows [center_begin, center_begin + count):
// F[k] += g_e for the row's own centre k, F[j] -= g_e for each neighbour j.
__global__ void forces_scatter_kernel(const int64_t* __restrict__ row_off, const int32_t* __restrict__ nbr,
                                      int64_t center_begin, int64_t count, int64_t N, const double* __restrict__ g,
                                      double* __restrict__ F) {
  const int64_t row0 = row_off[0];
  for (int64_t c = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; c < count; c += int64_t(gridDim.x) * blockDim.x) {
    const int64_t k = center_begin + c;
    double f[3] = {0.0, 0.0, 0.0};
    for (int64_t e = row_off[c] - row0; e < row_off[c + 1] - row0; ++e) {
      const int64_t j = nbr[e];
#pragma unroll
      for (int ax = 0; ax < 3; ++ax) {
        f[ax] += g[3 * e + ax];
        if (j >= 0 && j < N) atomicAdd(&F[3 * j + ax], -g[3 * e + ax]);
      }
    }
#pragma unroll
    for (int ax = 0; ax < 3; ++ax) atomicAdd(&F[3 * k + ax], f[ax]);
  }
}

int check_grad_tables(const y3b_ace_tables* t) {
  Y3B_CHECK_ARG(t != nullptr, "null tables");
  Y3B_CHECK_ARG(t->nmax >= 1 && t->nmax <= 16 && t->lmax >= 0 && t->lmax <= 6, "bad nmax / lmax");
  Y3B_CHECK_ARG(t->item_count >= 0 && t->phase_count >= 1, "bad table sizes");
  Y3B_CHECK_ARG(t->item_count == 0 || (t->items && t->item_coef && t->phases), "null item tables");
  return Y3B_OK;
}

}  // namespace
}  // namespace y3b

using namespace y3b;

extern "C" int y3b_ace_energy_grad(const y3b_ace_tables* tables, const void* A, int64_t atom_count,
                                   const int32_t* species, const double* weights, int64_t species_count,
                                   double* energy, void* dEdA, void* stream) {
  if (int rc = check_grad_tables(tables)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && species && weights && energy && dEdA && species_count > 0, "null pointer argument");
  const size_t smem = size_t(2) * size_t(tables->smem_entries + 2 * kGPad) * kGA * sizeof(double2);
  Y3B_CHECK_ARG(smem <= 200 * 1024, "bundle needs %lld bytes of shared memory for the adjoint (max 200 KB)",
                (long long)smem);
  Y3B_CUDA_TRY(cudaFuncSetAttribute(ace_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  const int64_t grid = (atom_count + kGA - 1) / kGA;
  Y3B_CHECK_ARG(grid < (int64_t(1) << 31), "too many atoms");
  ace_grad_kernel<<<int(grid), 32 * kGWarps, smem, as_stream(stream)>>>(
      *tables, static_cast<const double2*>(A), atom_count, species, weights, species_count, energy,
      static_cast<double2*>(dEdA));
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_ace_edge_grad(const double* positions, const int32_t* species, int64_t atom_count,
                                 int64_t center_begin, int64_t center_count, double box, const int64_t* row_offsets,
                                 const int32_t* neighbors, const double* species_prefactor, int64_t species_count,
                                 int64_t nmax, int64_t lmax, double cutoff, double lambda, const void* dEdA,
                                 double* edge_grad, int32_t* status, void* stream) {
  Y3B_CHECK_ARG(nmax >= 1 && nmax <= 16, "nmax must be in [1, 16]");
  Y3B_CHECK_ARG(center_begin >= 0 && center_count >= 0 && center_begin + center_count <= atom_count,
                "bad centre range");
  Y3B_CHECK_ARG(box > 0 && cutoff > 0, "box and cutoff must be positive");
  if (center_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(positions && species && row_offsets && species_prefactor && dEdA && edge_grad,
                "null pointer argument");
  const ShNorm nrm = make_sh_norm();
  const int grid = int(std::min<int64_t>((center_count + kEdgeWarps - 1) / kEdgeWarps, int64_t(kSMs) * 64));
  cudaStream_t s = as_stream(stream);
#define Y3B_EDGE_CASE(L)                                                                                    \
  case L:                                                                                                   \
    ace_edge_grad_kernel<L><<<grid, 32 * kEdgeWarps, 0, s>>>(                                               \
        positions, species, atom_count, center_begin, center_count, box, row_offsets, neighbors,            \
        species_prefactor, species_count, int(nmax), cutoff, lambda, nrm, static_cast<const double2*>(dEdA), \
        edge_grad, status);                                                                                  \
    break;
  switch (lmax) {
    Y3B_EDGE_CASE(0)
    Y3B_EDGE_CASE(1)
    Y3B_EDGE_CASE(2)
    Y3B_EDGE_CASE(3)
    Y3B_EDGE_CASE(4)
    default:
      return fail(Y3B_ERR_UNSUPPORTED, "ace_edge_grad: lmax %lld not built (0..4)", (long long)lmax);
  }
#undef Y3B_EDGE_CASE
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_forces_gather(const int64_t* row_offsets, const int32_t* neighbors, int64_t atom_count,
                                 const double* edge_grad, double* forces, int32_t* status, void* stream) {
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(row_offsets && forces, "null pointer argument");
  forces_gather_kernel<<<grid_for(atom_count, 128), 128, 0, as_stream(stream)>>>(row_offsets, neighbors, atom_count,
                                                                               edge_grad, forces, status);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_forces_scatter(const int64_t* row_offsets, const int32_t* neighbors, int64_t center_begin,
                                  int64_t center_count, int64_t atom_count, const double* edge_grad, double* forces,
                                  void* stream) {
  Y3B_CHECK_ARG(center_begin >= 0 && center_count >= 0 && center_begin + center_count <= atom_count,
                "bad centre range");
  if (center_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(row_offsets && edge_grad && forces, "null pointer argument");
  forces_scatter_kernel<<<grid_for(center_count, 128), 128, 0, as_stream(stream)>>>(
      row_offsets, neighbors, center_begin, center_count, atom_count, edge_grad, forces);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}
