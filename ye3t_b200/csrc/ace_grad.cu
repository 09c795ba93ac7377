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

// A CTA holds 16 atoms.  Values V ([entry][atom] complex, with zero entries
// before and after) and gradients G (real and imaginary planes, [entry][atom])
// live in shared memory.  Lanes l and l + 16 of a warp both work on atom l,
// each half-warp on its own item; the two items of a warp have the same shape
// (packing pairs them), so both halves follow one control flow.
//
// Gradients accumulate in registers and, for entries that leave a register
// window early, in a small per-lane staging area.  Class-0 items add each
// block's gradient to G once per item; the run paths (classes 1-3) keep a
// block's gradient over consecutive items of a lane and add it when the block
// changes.  The additions to G are batched compare-and-swaps: all old values
// are loaded, all swaps issued, and the ones that lost a race against another
// warp are added with red.shared.add.f64.
constexpr int kGA = 16;
#ifndef Y3B_RUN_WARPS
#define Y3B_RUN_WARPS 8
#endif
constexpr int kGWarps = 8;       // warps per CTA of the classes with symmetric slots
constexpr int kGWarpsRun = Y3B_RUN_WARPS;  // and of the four-block (A-only) classes

// Item classes of the adjoint (packing.grad_class assigns them); each class
// runs in its own kernel so that its item paths keep the register file.
// Every slot-class launch reloads A and redoes the symmetric slots of the
// phases it touches, so the slot items share two classes:
//   0: 1 and 2 blocks, 3 and 4 blocks with a register block of <= 3, and
//      anything the unrolled paths do not cover (generic path);
//   1: 3 blocks with a register block of 5 or 7;
//   2 / 3 (run classes): 4 blocks of A entries with a register block of 3 or
//      5 / 7 and prefix and last blocks of at most 7, no symmetric slots.
constexpr int kGradClasses = 4;
constexpr int kFirstRunClass = 2;

template <int CLS>
struct ClassWarps {
  static constexpr int value = CLS >= kFirstRunClass ? kGWarpsRun : kGWarps;
};
constexpr int kGPad = 16;
constexpr int kStage = 14;     // staged gradient entries per lane (two blocks of <= 7)
constexpr int kStageRun = 21;  // the same for the four-block run path (three blocks of <= 7)
#ifndef Y3B_GRAD_BATCH
#define Y3B_GRAD_BATCH 2
#endif

// This lane's data in shared memory.  V and the staging area are read and
// written with ordinary loads and stores (V is read-only during the item walk,
// the staging area is private to the lane), so the compiler schedules them
// freely; G is only touched by the compare-and-swap batches, through
// shared-window (32-bit) byte addresses.
struct Ctx {
  const double2* V;  // V[e * kGA]: entry e of this lane's atom
  uint32_t Gr, Gi;   // its gradient planes, entry e at + e * kGA * 8
  double2* stage;    // stage[k * 32]: this lane's staged entry k
};

__device__ __forceinline__ double2 vat(const Ctx& c, int e) { return c.V[e * kGA]; }

__device__ __forceinline__ double2 cscale(double s, double2 v) { return make_double2(s * v.x, s * v.y); }

__device__ __forceinline__ unsigned long long dbits(double x) {
  return static_cast<unsigned long long>(__double_as_longlong(x));
}

__device__ __forceinline__ unsigned long long lds64(uint32_t a) {
  unsigned long long v;
  asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(a));
  return v;
}

__device__ __forceinline__ unsigned long long cas64(uint32_t a, unsigned long long cmp, unsigned long long val) {
  unsigned long long old;
  asm volatile("atom.shared.cas.b64 %0, [%1], %2, %3;" : "=l"(old) : "r"(a), "l"(cmp), "l"(val));
  return old;
}

__device__ __forceinline__ void red_add64(uint32_t a, double v) {
  asm volatile("red.shared.add.f64 [%0], %1;" ::"r"(a), "d"(v));
}

// G[base + STEP * k] += v[k] for K0 <= k < K0 + NB, lo <= k < hi: loads the
// old values, then issues every compare-and-swap at once; the few that lost a
// race against another warp are redone as single atomic additions.  The loads
// and swaps are volatile asm, so successive batches stay in program order.
template <int NB, int STEP, int K0, int N>
__device__ __forceinline__ void g_add_batch_lanes(uint32_t ar, uint32_t ai, int lo, int hi, const double2 (&v)[N]) {
  constexpr int kStride = STEP * kGA * 8;
  unsigned long long o[2 * NB];
#pragma unroll
  for (int b = 0; b < 2 * NB; ++b) {
    const int k = K0 + (b >> 1);
    const double x = k < N ? ((b & 1) ? v[k < N ? k : 0].y : v[k < N ? k : 0].x) : 0.0;
    if (k < N && k >= lo && k < hi && x != 0.0) o[b] = lds64(((b & 1) ? ai : ar) + k * kStride);
  }
#pragma unroll
  for (int b = 0; b < 2 * NB; ++b) {
    const int k = K0 + (b >> 1);
    const double x = k < N ? ((b & 1) ? v[k < N ? k : 0].y : v[k < N ? k : 0].x) : 0.0;
    if (k < N && k >= lo && k < hi && x != 0.0) {
      const uint32_t a = ((b & 1) ? ai : ar) + k * kStride;
      const unsigned long long want = dbits(__longlong_as_double(static_cast<long long>(o[b])) + x);
      o[b] = cas64(a, o[b], want) ^ o[b];  // 0 when the swap took effect
    }
  }
#pragma unroll
  for (int b = 0; b < 2 * NB; ++b) {
    const int k = K0 + (b >> 1);
    const double x = k < N ? ((b & 1) ? v[k < N ? k : 0].y : v[k < N ? k : 0].x) : 0.0;
    if (k < N && k >= lo && k < hi && x != 0.0 && o[b] != 0) red_add64(((b & 1) ? ai : ar) + k * kStride, x);
  }
}

template <int NB, int STEP, int K0, int N>
__device__ __forceinline__ void g_add_batch(const Ctx& c, uint32_t ar, uint32_t ai, int lo, int hi,
                                            const double2 (&v)[N]) {
  g_add_batch_lanes<NB, STEP, K0, N>(ar, ai, lo, hi, v);
}

constexpr int kBatch = Y3B_GRAD_BATCH;

template <int STEP, int K0, int N>
struct GAddChunks {
  static __device__ __forceinline__ void run(const Ctx& c, uint32_t ar, uint32_t ai, int lo, int hi,
                                             const double2 (&v)[N]) {
    g_add_batch<kBatch, STEP, K0, N>(c, ar, ai, lo, hi, v);
    if constexpr (K0 + kBatch < N) GAddChunks<STEP, K0 + kBatch, N>::run(c, ar, ai, lo, hi, v);
  }
};

// G[base + STEP * k] += v[k] for lo <= k < hi (zero parts are skipped).
template <int N, int STEP>
__device__ __forceinline__ void g_add(const Ctx& c, int base, int lo, int hi, const double2 (&v)[N]) {
  const uint32_t ar = c.Gr + base * (kGA * 8), ai = c.Gi + base * (kGA * 8);
  GAddChunks<STEP, 0, N>::run(c, ar, ai, lo, hi, v);
}

__device__ __forceinline__ void g_add1(const Ctx& c, int e, double2 v) {
  const double2 a[1] = {v};
  g_add<1, 1>(c, e, 0, 1, a);
}


// G[base + STEP * k] += staged entry off + k for lo <= k < hi (< NMAX),
// kBatch entries at a time.
template <int STEP, int NMAX = kStage>
__device__ __forceinline__ void stage_flush_impl(const Ctx& c, int base, int off, int lo, int hi) {
  const uint32_t ar = c.Gr + base * (kGA * 8), ai = c.Gi + base * (kGA * 8);
#pragma unroll
  for (int k0 = 0; k0 < NMAX; k0 += kBatch) {
    if (k0 < hi && k0 + kBatch > lo) {
      double2 v[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int k = k0 + u;
        v[u] = (k < NMAX && k >= lo && k < hi) ? c.stage[(off + k) * 32] : make_double2(0.0, 0.0);
      }
      g_add_batch<kBatch, STEP, 0, kBatch>(c, ar + STEP * k0 * (kGA * 8), ai + STEP * k0 * (kGA * 8), lo - k0,
                                           hi - k0, v);
    }
  }
}

__device__ __forceinline__ void stage_flush(const Ctx& c, int base, int lo, int hi) {
  stage_flush_impl<1>(c, base, 0, lo, hi);
}
__device__ __forceinline__ void stage_flush_off(const Ctx& c, int base, int off, int lo, int hi) {
  stage_flush_impl<1>(c, base, off, lo, hi);
}

// Staged accumulation: entry k of this lane's staging area += v (private to
// the lane, so a plain read-modify-write).
__device__ __forceinline__ void stage_acc(const Ctx& c, int k, double2 v) {
  double2* a = c.stage + k * 32;
  *a = add(*a, v);
}

__device__ __forceinline__ void stage_zero(const Ctx& c, int lo, int hi) {
#pragma unroll 1
  for (int k = lo; k < hi; ++k) c.stage[k * 32] = make_double2(0.0, 0.0);
}

// The register block is walked in chunks of CH indices j (runtime width jn <=
// CH); the adjoint's item classes each run in their own kernel with CH equal
// to the class's register-block size, so a chunk is the whole block.

// Readout-weighted coefficients j0 .. j0 + CH - 1 of a row (zero past jn):
// wc[u] = w0 C[j0 + u, 0] + w1 C[j0 + u, 1]; rows are 16-byte aligned, so for
// even j0 single-component pairs are read with 16-byte loads.
template <int CH>
__device__ __forceinline__ void wchunk(const double* __restrict__ crow, int nc, int j0, int jn, double w0, double w1,
                                       double (&wc)[CH]) {
  const double2* c2 = reinterpret_cast<const double2*>(crow);
  if (nc == 2) {
#pragma unroll
    for (int u = 0; u < CH; ++u) {
      const double2 cc = u < jn ? __ldg(c2 + j0 + u) : make_double2(0.0, 0.0);
      wc[u] = fma(w1, cc.y, w0 * cc.x);
    }
  } else if ((j0 & 1) == 0) {
#pragma unroll
    for (int u = 0; u < CH; u += 2) {
      const double2 cc = u < jn ? __ldg(c2 + (j0 + u) / 2) : make_double2(0.0, 0.0);
      wc[u] = w0 * cc.x;
      if (u + 1 < CH) wc[u + 1] = u + 1 < jn ? w0 * cc.y : 0.0;
    }
  } else {
#pragma unroll
    for (int u = 0; u < CH; ++u) wc[u] = u < jn ? w0 * __ldg(crow + j0 + u) : 0.0;
  }
}

__device__ __forceinline__ double adj1(const Ctx& c, const Item& it, int nc, const double* __restrict__ coef,
                                       double w0, double w1, bool mute) {
  const double* cr = coef + it.coef;
  const double wc = nc == 2 ? fma(w1, __ldg(cr + 1), w0 * __ldg(cr)) : w0 * __ldg(cr);
  if (!mute) g_add1(c, it.b0 + it.K, make_double2(wc, 0.0));
  return wc * vat(c, it.b0 + it.K).x;
}

// Two blocks (register block s of ds indices, last block l = K - j): one
// row.  Per chunk of CH indices, gs and gl are added to G from registers.
template <int CH>
__device__ __forceinline__ double adj2(const Ctx& c, const Item& it, int ds, int nc, const double* __restrict__ coef,
                                       double w0, double w1, bool mute) {
  double e = 0.0;
  const int bs = it.b0, bl = it.b1, K = it.K, dl = it.dl;
  const double* cr = coef + it.coef;
#pragma unroll 1
  for (int j0 = 0; j0 < ds; j0 += CH) {
    const int jn = min(CH, ds - j0);
    double wc[CH];
    wchunk<CH>(cr, nc, j0, jn, w0, w1, wc);
    double2 gs[CH], gl[CH];
#pragma unroll
    for (int u = 0; u < CH; ++u) {
      gs[u] = gl[u] = make_double2(0.0, 0.0);
      if (u < jn) {
        // out-of-block last indices read finite neighbours; their coefficient is 0
        const double2 xs = vat(c, bs + j0 + u), xl = vat(c, bl + K - j0 - u);
        e += wc[u] * (xs.x * xl.x - xs.y * xl.y);
        gs[u] = cscale(wc[u], xl);
        gl[u] = cscale(wc[u], xs);
      }
    }
    if (!mute) {
      g_add<CH, 1>(c, bs + j0, 0, jn, gs);
      // gl[u] belongs to last-block index K - j0 - u
      g_add<CH, -1>(c, bl + K - j0, max(0, K - j0 - dl + 1), min(jn, K - j0 + 1), gl);
    }
  }
  return e;
}

// Three blocks: rows i0 (prefix block 0), register block s, last block
// l = K - i0 - j (dl <= kStage, gl accumulates in the staging area).  The
// prefix gradient of a row is T_i0, added to G per row and chunk.
template <int CH>
__device__ __forceinline__ double adj3(const Ctx& c, const Item& it, int ds, int nc, const double* __restrict__ coef,
                                       double w0, double w1, bool mute) {
  double e = 0.0;
  const int rw = nc == 2 ? 2 * ds : ((ds + 1) & ~1);
  const int b0 = it.b0, bs = it.b1, bl = it.b2, K = it.K, dl = it.dl;
  const int r_lo = max(0, K - (ds - 1) - (dl - 1)), r_hi = min(it.d0 - 1, K);
  if (r_lo > r_hi) return e;
  const double* cb = coef + it.coef;
  stage_zero(c, 0, dl);
#pragma unroll 1
  for (int j0 = 0; j0 < ds; j0 += CH) {
    const int jn = min(CH, ds - j0);
    double2 vs[CH], gs[CH];
#pragma unroll
    for (int u = 0; u < CH; ++u) {
      vs[u] = u < jn ? vat(c, bs + j0 + u) : make_double2(0.0, 0.0);
      gs[u] = make_double2(0.0, 0.0);
    }
    // w[u] belongs to last-block index K - r - j0 - u (moves by one per row)
    double2 w[CH];
#pragma unroll
    for (int u = 0; u < CH; ++u) w[u] = make_double2(0.0, 0.0);
#pragma unroll 1
    for (int r = r_lo; r <= r_hi; ++r) {
      double wc[CH];
      wchunk<CH>(cb + r * rw, nc, j0, jn, w0, w1, wc);
      const double2 x0 = vat(c, b0 + r);
      double2 T = make_double2(0.0, 0.0);
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        // out-of-block last indices read finite neighbours; their coefficient is 0
        const double2 vl = vat(c, bl + K - r - j0 - u);
        cmac(T, wc[u], mul(vs[u], vl));
        const double2 xw = cscale(wc[u], x0);
        cfma(gs[u], xw, vl);
        cfma(w[u], xw, vs[u]);
      }
      e += x0.x * T.x - x0.y * T.y;
      if (!mute) g_add1(c, b0 + r, T);
      const int kf = K - r - j0;
      if (kf >= 0 && kf < dl) stage_acc(c, kf, w[0]);
#pragma unroll
      for (int u = 0; u + 1 < CH; ++u) w[u] = w[u + 1];
      w[CH - 1] = make_double2(0.0, 0.0);
    }
#pragma unroll
    for (int u = 0; u + 1 < CH; ++u) {
      const int k = K - r_hi - 1 - j0 - u;
      if (k >= 0 && k < dl) stage_acc(c, k, w[u]);
    }
    if (!mute) g_add<CH, 1>(c, bs + j0, 0, jn, gs);
  }
  if (!mute) stage_flush(c, bl, 0, dl);
  return e;
}

// Three-block item (register block of ds <= CH indices) accumulating into
// state that persists over a run of items: g_s in gs, g_last staged at
// [0, dl).  The prefix gradient T_r of a row is added to G per row (a muted
// lane has zero weights and adds zeros).
template <int CH, int NG>
__device__ __forceinline__ double adj3_acc(const Ctx& c, const Item& it, int ds, int nc,
                                           const double* __restrict__ coef, double w0, double w1,
                                           double2 (&gs)[NG]) {
  static_assert(CH <= NG, "register-block gradient shorter than the block");
  double e = 0.0;
  const int rw = nc == 2 ? 2 * ds : ((ds + 1) & ~1);
  const int b0 = it.b0, bs = it.b1, bl = it.b2, K = it.K, dl = it.dl;
  const int r_lo = max(0, K - (ds - 1) - (dl - 1)), r_hi = min(it.d0 - 1, K);
  if (r_lo > r_hi) return e;
  const double* cb = coef + it.coef;
  double2 vs[CH], w[CH];
#pragma unroll
  for (int u = 0; u < CH; ++u) {
    vs[u] = u < ds ? vat(c, bs + u) : make_double2(0.0, 0.0);
    w[u] = make_double2(0.0, 0.0);
  }
  // w[u] belongs to last-block index K - r - u (moves by one per row)
#pragma unroll 1
  for (int r = r_lo; r <= r_hi; ++r) {
    double wc[CH];
    wchunk<CH>(cb + r * rw, nc, 0, ds, w0, w1, wc);
    const double2 x0 = vat(c, b0 + r);
    double2 T = make_double2(0.0, 0.0);
#pragma unroll
    for (int u = 0; u < CH; ++u) {
      // out-of-block last indices read finite neighbours; their coefficient is 0
      const double2 vl = vat(c, bl + K - r - u);
      cmac(T, wc[u], mul(vs[u], vl));
      const double2 xw = cscale(wc[u], x0);
      cfma(gs[u], xw, vl);
      cfma(w[u], xw, vs[u]);
    }
    e += x0.x * T.x - x0.y * T.y;
    g_add1(c, b0 + r, T);
    const int kf = K - r;
    if (kf >= 0 && kf < dl) stage_acc(c, kf, w[0]);
#pragma unroll
    for (int u = 0; u + 1 < CH; ++u) w[u] = w[u + 1];
    w[CH - 1] = make_double2(0.0, 0.0);
  }
#pragma unroll
  for (int u = 0; u + 1 < CH; ++u) {
    const int k = K - r_hi - 1 - u;
    if (k >= 0 && k < dl) stage_acc(c, k, w[u]);
  }
  return e;
}

// A warp's sorted run of three-block item pairs [g, ge) inside one phase
// (class 1: register blocks of 5 or 7 indices).  As in the four-block run
// path, the register block's gradient stays in registers and the last
// block's in the staging area until the next item's block differs.  An item
// outside the path's bounds is skipped and reported in *bad.
__device__ __forceinline__ double adj3_run(const Ctx& c, const int2* __restrict__ pairs, int g, int ge, int grp,
                                           const int4* __restrict__ items, const double* __restrict__ coef,
                                           const double* __restrict__ wz, bool& bad) {
  constexpr int NG = 7;
  double e = 0.0;
  double2 gs[NG];
#pragma unroll
  for (int u = 0; u < NG; ++u) gs[u] = make_double2(0.0, 0.0);
  int ps = -1, ns = 0, pl = -1, nl = 0;
#pragma unroll 1
  for (; g < ge; ++g) {
    const int2 ig = __ldg(pairs + g);
    if (ig.x < 0) continue;  // null pair padding a run (the whole warp skips it)
    const int mine = grp == 0 ? ig.x : ig.y;
    const bool mute = mine < 0;
    const Item it = load_item(items, mute ? ig.x : mine);
    const int ds = 2 * ((it.sel >> 1) % 7) + 1, B = (it.sel >> 1) / 7 + 1;
    if (B != 3 || it.dl > kStage || (ds != 5 && ds != 7)) {
      bad = true;
      continue;
    }
    const double w0 = mute ? 0.0 : __ldg(wz + it.f0);
    const double w1 = (!mute && it.f1 >= 0) ? __ldg(wz + it.f1) : 0.0;
    if (it.b1 != ps || ds != ns) {
      if (ps >= 0) g_add<NG, 1>(c, ps, 0, ns, gs);
#pragma unroll
      for (int u = 0; u < NG; ++u) gs[u] = make_double2(0.0, 0.0);
      ps = it.b1;
      ns = ds;
    }
    if (it.b2 != pl || it.dl != nl) {
      if (pl >= 0) stage_flush_impl<1, kStage>(c, pl, 0, 0, nl);
      stage_zero(c, 0, it.dl);
      pl = it.b2;
      nl = it.dl;
    }
    const int nc = (it.sel & 1) + 1;
    if (ds == 5)
      e += adj3_acc<5>(c, it, ds, nc, coef, w0, w1, gs);
    else
      e += adj3_acc<7>(c, it, ds, nc, coef, w0, w1, gs);
  }
  if (ps >= 0) g_add<NG, 1>(c, ps, 0, ns, gs);
  if (pl >= 0) stage_flush_impl<1, kStage>(c, pl, 0, 0, nl);
  return e;
}

// Four blocks: rows (i0, i1) of prefix blocks 0 and 1 (d0 <= d1 <= 7), the
// register block s and the last block l = K - S - j with S = i0 + i1 (dl <=
// 14).  Rows of one anti-diagonal S share q_j = vs_j vl_{K-S-j}.  Two passes
// over the anti-diagonals, each chunk of j in turn:
//   A: T per row; g0[i0] += x1 T and g1[i1] += x0 T accumulate in the
//      staging area ([0, 7) and [7, 14));
//   B: R_j = sum over the diagonal's rows of c_j x0 x1; gs[j] += R_j vl
//      (registers, per chunk) and gl[K - S - j] += R_j vs_j (staged at [0, dl)).
template <int CH>
__device__ __forceinline__ double adj4(const Ctx& c, const Item& it, int ds, int nc, const double* __restrict__ coef,
                                       double w0, double w1, bool mute) {
  double e = 0.0;
  const int rw = nc == 2 ? 2 * ds : ((ds + 1) & ~1);
  const int b0 = it.b0, b1 = it.b1, bs = it.b2, bl = it.b3;
  const int d0 = it.d0, d1 = it.d1, dl = it.dl, K = it.K;
  const int s_lo = max(0, K - (ds - 1) - (dl - 1)), s_hi = min(d0 + d1 - 2, K);
  if (s_lo > s_hi) return e;
  const double* cb = coef + it.coef;
  stage_zero(c, 0, d0);
  stage_zero(c, 7, 7 + d1);
#pragma unroll 1
  for (int j0 = 0; j0 < ds; j0 += CH) {
    const int jn = min(CH, ds - j0);
    double2 vs[CH];
#pragma unroll
    for (int u = 0; u < CH; ++u) vs[u] = u < jn ? vat(c, bs + j0 + u) : make_double2(0.0, 0.0);
#pragma unroll 1
    for (int S = s_lo; S <= s_hi; ++S) {
      double2 q[CH];
#pragma unroll
      for (int u = 0; u < CH; ++u) q[u] = mul(vs[u], vat(c, bl + K - S - j0 - u));
      const int i0a = max(0, S - (d1 - 1)), i0b = min(d0 - 1, S);
#pragma unroll 1
      for (int i0 = i0a; i0 <= i0b; ++i0) {
        const int i1 = S - i0;
        double wc[CH];
        wchunk<CH>(cb + (i0 * d1 + i1) * rw, nc, j0, jn, w0, w1, wc);
        double2 T = make_double2(0.0, 0.0), To = T;  // even and odd u: two independent chains
#pragma unroll
        for (int u = 0; u < CH; ++u) cmac((u & 1) ? To : T, wc[u], q[u]);
        T = add(T, To);
        const double2 x0 = vat(c, b0 + i0), x1 = vat(c, b1 + i1);
        const double2 x01 = mul(x0, x1);
        e += x01.x * T.x - x01.y * T.y;
        stage_acc(c, i0, mul(x1, T));
        stage_acc(c, 7 + i1, mul(x0, T));
      }
    }
  }
  if (!mute) {
    stage_flush(c, b0, 0, d0);
    stage_flush_off(c, b1, 7, 0, d1);
  }
  stage_zero(c, 0, dl);
#pragma unroll 1
  for (int j0 = 0; j0 < ds; j0 += CH) {
    const int jn = min(CH, ds - j0);
    double2 vs[CH], gs[CH];
#pragma unroll
    for (int u = 0; u < CH; ++u) {
      vs[u] = u < jn ? vat(c, bs + j0 + u) : make_double2(0.0, 0.0);
      gs[u] = make_double2(0.0, 0.0);
    }
    // w[u] belongs to last-block index K - S - j0 - u; after diagonal S no
    // later one reaches index K - S - j0, which is added to the staging area
    double2 w[CH];
#pragma unroll
    for (int u = 0; u < CH; ++u) w[u] = make_double2(0.0, 0.0);
#pragma unroll 1
    for (int S = s_lo; S <= s_hi; ++S) {
      double2 R[CH];
#pragma unroll
      for (int u = 0; u < CH; ++u) R[u] = make_double2(0.0, 0.0);
      const int i0a = max(0, S - (d1 - 1)), i0b = min(d0 - 1, S);
#pragma unroll 1
      for (int i0 = i0a; i0 <= i0b; ++i0) {
        const int i1 = S - i0;
        double wc[CH];
        wchunk<CH>(cb + (i0 * d1 + i1) * rw, nc, j0, jn, w0, w1, wc);
        const double2 x01 = mul(vat(c, b0 + i0), vat(c, b1 + i1));
#pragma unroll
        for (int u = 0; u < CH; ++u) cmac(R[u], wc[u], x01);
      }
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        cfma(gs[u], R[u], vat(c, bl + K - S - j0 - u));
        cfma(w[u], R[u], vs[u]);
      }
      const int kf = K - S - j0;
      if (kf >= 0 && kf < dl) stage_acc(c, kf, w[0]);
#pragma unroll
      for (int u = 0; u + 1 < CH; ++u) w[u] = w[u + 1];
      w[CH - 1] = make_double2(0.0, 0.0);
    }
#pragma unroll
    for (int u = 0; u + 1 < CH; ++u) {
      const int k = K - s_hi - 1 - j0 - u;
      if (k >= 0 && k < dl) stage_acc(c, k, w[u]);
    }
    if (!mute) g_add<CH, 1>(c, bs + j0, 0, jn, gs);
  }
  if (!mute) stage_flush(c, bl, 0, dl);
  return e;
}

// Four-block item, register block of exactly CH indices, accumulating into
// state that persists over a run of items: g0 and g1 in staging regions
// [0, 7) and [7, 14), g_last in [14, 21), g_s in gs.  One pass over the
// anti-diagonals S: q_u = vs_u vl[K-S-u]; per row T = sum_u c_u q_u gives the
// energy and the prefix gradients, and R_u += c_u x0 x1; per diagonal
// gs_u += R_u vl[K-S-u] and g_last[K-S-u] += R_u vs_u (through a window that
// moves by one per diagonal).
template <int CH, int NG>
__device__ __forceinline__ double adj4_body(const Ctx& c, const Item& it, int nc, const double* __restrict__ coef,
                                            double w0, double w1, double2 (&gs)[NG]) {
  static_assert(CH <= NG, "register-block gradient shorter than the block");
  double e = 0.0;
  constexpr int rw_1 = (CH + 1) & ~1;
  const int rw = nc == 2 ? 2 * CH : rw_1;
  const int b0 = it.b0, b1 = it.b1, bs = it.b2, bl = it.b3;
  const int d0 = it.d0, d1 = it.d1, dl = it.dl, K = it.K;
  const int s_lo = max(0, K - (CH - 1) - (dl - 1)), s_hi = min(d0 + d1 - 2, K);
  if (s_lo > s_hi) return e;
  const double* cb = coef + it.coef;
  // register-block values: held in registers for the smaller blocks, read
  // from shared memory at each use for the 7-index block (register budget)
  constexpr int NS = CH <= 5 ? CH : 1;
  double2 vs[NS] = {}, w[CH];
  auto vsu = [&](int u) { return CH <= 5 ? vs[u < NS ? u : 0] : vat(c, bs + u); };
#pragma unroll
  for (int u = 0; u < CH; ++u) {
    if (CH <= 5) vs[u < NS ? u : 0] = vat(c, bs + u);
    w[u] = make_double2(0.0, 0.0);
  }
#pragma unroll 1
  for (int S = s_lo; S <= s_hi; ++S) {
    // last-block values of the diagonal, held over its rows
    double2 vl[CH], q[CH], R[CH];
#pragma unroll
    for (int u = 0; u < CH; ++u) {
      const double2 v = vat(c, bl + K - S - u);  // out-of-block indices read finite neighbours; their coefficient is 0
      vl[u] = v;
      q[u] = mul(vsu(u), v);
      R[u] = make_double2(0.0, 0.0);
    }
    const int i0a = max(0, S - (d1 - 1)), i0b = min(d0 - 1, S);
#pragma unroll 1
    for (int i0 = i0a; i0 <= i0b; ++i0) {
      const int i1 = S - i0;
      double wc[CH];
      wchunk<CH>(cb + (i0 * d1 + i1) * rw, nc, 0, CH, w0, w1, wc);
      double2 T = make_double2(0.0, 0.0), To = T;  // even and odd u: two independent chains
#pragma unroll
      for (int u = 0; u < CH; ++u) cmac((u & 1) ? To : T, wc[u], q[u]);
      T = add(T, To);
      const double2 x0 = vat(c, b0 + i0), x1 = vat(c, b1 + i1);
      const double2 x01 = mul(x0, x1);
      e += x01.x * T.x - x01.y * T.y;
      stage_acc(c, i0, mul(x1, T));
      stage_acc(c, 7 + i1, mul(x0, T));
#pragma unroll
      for (int u = 0; u < CH; ++u) cmac(R[u], wc[u], x01);
    }
#pragma unroll
    for (int u = 0; u < CH; ++u) {
      cfma(gs[u], R[u], vl[u]);
      cfma(w[u], R[u], vsu(u));
    }
    // w[u] belongs to last-block index K - S - u; no later diagonal reaches K - S
    const int kf = K - S;
    if (kf >= 0 && kf < dl) stage_acc(c, 14 + kf, w[0]);
#pragma unroll
    for (int u = 0; u + 1 < CH; ++u) w[u] = w[u + 1];
    w[CH - 1] = make_double2(0.0, 0.0);
  }
#pragma unroll
  for (int u = 0; u + 1 < CH; ++u) {
    const int k = K - s_hi - 1 - u;
    if (k >= 0 && k < dl) stage_acc(c, 14 + k, w[u]);
  }
  return e;
}

// A warp's contiguous run of four-block item pairs [g, ge) (run classes 2, 3;
// register blocks of 3 or 5 indices in class 2, 7 in class 3).  Packing sorts
// each shape's items by (register block, last block, prefix blocks) and gives
// each half-warp a sorted half, so consecutive items of a lane mostly share
// blocks: a target's gradient is added to G only when the next item's block
// differs (a muted lane adds zeros, which changes nothing).  Both half-warps
// run items of one shape, so the per-item branches are warp-uniform.  An item
// outside the run path's bounds (blocks longer than the 7-entry staging
// windows, another register block) is skipped and reported in *bad.
template <int CLS>
__device__ __forceinline__ double adj4_run(const Ctx& c, const int2* __restrict__ pairs, int g, int ge, int grp,
                                           const int4* __restrict__ items, const double* __restrict__ coef,
                                           const double* __restrict__ wz, bool& bad) {
  constexpr bool kSmall = CLS == kFirstRunClass;  // register blocks of 3 or 5
  constexpr int NG = kSmall ? 5 : 7;
  double e = 0.0;
  double2 gs[NG];
#pragma unroll
  for (int u = 0; u < NG; ++u) gs[u] = make_double2(0.0, 0.0);
  int p0 = -1, p1 = -1, ps = -1, pl = -1, n0 = 0, n1 = 0, ns = 0, nl = 0;
#pragma unroll 1
  for (; g < ge; ++g) {
    const int2 ig = __ldg(pairs + g);
    if (ig.x < 0) continue;  // null pair padding a run (the whole warp skips it)
    const int mine = grp == 0 ? ig.x : ig.y;
    const bool mute = mine < 0;
    const Item it = load_item(items, mute ? ig.x : mine);
    const int ds = 2 * ((it.sel >> 1) % 7) + 1;
    if (it.d0 > 7 || it.d1 > 7 || it.dl > 7 || (kSmall ? (ds != 3 && ds != 5) : ds != 7)) {
      bad = true;
      continue;
    }
    const double w0 = mute ? 0.0 : __ldg(wz + it.f0);
    const double w1 = (!mute && it.f1 >= 0) ? __ldg(wz + it.f1) : 0.0;
    if (it.b0 != p0) {
      if (p0 >= 0) stage_flush_impl<1, 7>(c, p0, 0, 0, n0);
      stage_zero(c, 0, it.d0);
      p0 = it.b0;
      n0 = it.d0;
    }
    if (it.b1 != p1) {
      if (p1 >= 0) stage_flush_impl<1, 7>(c, p1, 7, 0, n1);
      stage_zero(c, 7, 7 + it.d1);
      p1 = it.b1;
      n1 = it.d1;
    }
    if (it.b2 != ps || (kSmall && ds != ns)) {
      if (ps >= 0) g_add<NG, 1>(c, ps, 0, kSmall ? ns : NG, gs);
#pragma unroll
      for (int u = 0; u < NG; ++u) gs[u] = make_double2(0.0, 0.0);
      ps = it.b2;
      ns = ds;
    }
    if (it.b3 != pl) {
      if (pl >= 0) stage_flush_impl<1, 7>(c, pl, 14, 0, nl);
      stage_zero(c, 14, 14 + it.dl);
      pl = it.b3;
      nl = it.dl;
    }
    const int nc = (it.sel & 1) + 1;
    if (kSmall && ds == 3)
      e += adj4_body<3>(c, it, nc, coef, w0, w1, gs);
    else
      e += adj4_body<NG>(c, it, nc, coef, w0, w1, gs);
  }
  if (p0 >= 0) stage_flush_impl<1, 7>(c, p0, 0, 0, n0);
  if (p1 >= 0) stage_flush_impl<1, 7>(c, p1, 7, 0, n1);
  if (ps >= 0) g_add<NG, 1>(c, ps, 0, kSmall ? ns : NG, gs);
  if (pl >= 0) stage_flush_impl<1, 7>(c, pl, 14, 0, nl);
  return e;
}

// Any item shape, one tuple at a time with single additions (for shapes the
// unrolled paths do not cover: wide register blocks, long last blocks).
__device__ __noinline__ double adj_generic(const Ctx c, const Item it, int B, int DS, int NC,
                                           const double* __restrict__ coef, double w0, double w1, bool mute) {
  double e = 0.0;
  const int RW = NC == 2 ? 2 * DS : ((DS + 1) & ~1);
  const int n0 = B >= 3 ? it.d0 : 1, n1 = B == 4 ? it.d1 : 1;
  const int bs = B == 2 ? it.b0 : (B == 3 ? it.b1 : it.b2);
  const int bl = B == 2 ? it.b1 : (B == 3 ? it.b2 : it.b3);
  const double2 one = make_double2(1.0, 0.0);
  for (int i0 = 0; i0 < n0; ++i0) {
    for (int i1 = 0; i1 < n1; ++i1) {
      const int row = B == 4 ? i0 * it.d1 + i1 : (B == 3 ? i0 : 0);
      const double* cr = coef + it.coef + row * RW;
      const double2 x0 = B >= 3 ? vat(c, it.b0 + i0) : one;
      const double2 x1 = B == 4 ? vat(c, it.b1 + i1) : one;
      const double2 p01 = mul(x0, x1);
      for (int j = 0; j < DS; ++j) {
        const int k = it.K - i0 - i1 - j;
        if (k < 0 || k >= it.dl) continue;
        const double wc = NC == 2 ? fma(w1, __ldg(cr + 2 * j + 1), w0 * __ldg(cr + 2 * j)) : w0 * __ldg(cr + j);
        if (wc == 0.0) continue;
        const double2 xs = vat(c, bs + j), xl = vat(c, bl + k);
        const double2 psl = mul(xs, xl);
        e += wc * (p01.x * psl.x - p01.y * psl.y);
        if (mute) continue;
        if (B >= 3) g_add1(c, it.b0 + i0, cscale(wc, mul(x1, psl)));
        if (B == 4) g_add1(c, it.b1 + i1, cscale(wc, mul(x0, psl)));
        g_add1(c, bs + j, cscale(wc, mul(p01, xl)));
        g_add1(c, bl + k, cscale(wc, mul(p01, xs)));
      }
    }
  }
  return e;
}

template <int CLS>
__device__ __forceinline__ double adj_class(const Ctx& c, const Item& it, const double* __restrict__ coef,
                                            double w0, double w1, bool mute) {
  const int nc = (it.sel & 1) + 1, ds = 2 * ((it.sel >> 1) % 7) + 1, B = (it.sel >> 1) / 7 + 1;
  const bool fits3 = B == 3 && it.dl <= kStage;
  const bool fits4 = B == 4 && it.d0 <= 7 && it.d1 <= 7 && it.dl <= kStage;
  static_assert(CLS == 0, "class 0 only (class 1 and the run classes walk sorted runs)");
  if (B == 1) return adj1(c, it, nc, coef, w0, w1, mute);
  if (B == 2) return adj2<8>(c, it, ds, nc, coef, w0, w1, mute);
  if (fits3 && ds <= 3) return adj3<3>(c, it, ds, nc, coef, w0, w1, mute);
  if (fits4 && ds <= 3) return adj4<3>(c, it, ds, nc, coef, w0, w1, mute);
  return adj_generic(c, it, B, ds, nc, coef, w0, w1, mute);
}

// Fill and pull-back tables of the symmetric slots.  At a phase change no
// item is running, so the per-lane staging area is free: the CTA copies the
// tables there (about 16 KB for l_max 3) and the fill and the pull read them
// from shared memory instead of through chains of L2 reads; tables larger
// than the staging area are read from global memory.
struct SymTabs {
  const int4* outs;     // [so]: l^2, term begin, term end
  const uint32_t* fac;  // [nterm] 4 x u8 factors
  const double* co;     // [nterm]
  int nterm;
  const int32_t* goff;  // [W + 1]
  const int2* gidx;     // [T]: output, 4 x u8 remaining factors
  const double* gco;    // [T]
};

__device__ __forceinline__ int sym_term_total(const y3b_ace_tables& t) { return int(t.sym_term_count); }

__device__ __forceinline__ SymTabs sym_tabs_global(const y3b_ace_tables& t, int nterm) {
  return SymTabs{reinterpret_cast<const int4*>(t.sym_outputs), t.sym_term_factors, t.sym_term_coeff, nterm,
                 t.sym_grad_offsets, reinterpret_cast<const int2*>(t.sym_grad_index), t.sym_grad_coeff};
}

__host__ __device__ __forceinline__ size_t sym_tabs_bytes(int so, int nterm, int W, int64_t T) {
  const size_t a = size_t(16) * so, b = (size_t(4) * nterm + 15) & ~size_t(15), c = size_t(8) * nterm;
  const size_t d = (size_t(4) * (W + 1) + 15) & ~size_t(15);
  return a + b + ((c + 15) & ~size_t(15)) + d + size_t(16) * T;
}

// All threads copy; the caller synchronises before reading.  base is 16-byte aligned.
__device__ __forceinline__ SymTabs sym_tabs_stage(const y3b_ace_tables& t, char* base, int nterm, int W) {
  const int so = int(t.sym_output_count), T = int(t.sym_grad_count);
  int4* outs = reinterpret_cast<int4*>(base);
  uint32_t* fac = reinterpret_cast<uint32_t*>(base + size_t(16) * so);
  double* co = reinterpret_cast<double*>(reinterpret_cast<char*>(fac) + ((size_t(4) * nterm + 15) & ~size_t(15)));
  int32_t* goff = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(co) + ((size_t(8) * nterm + 15) & ~size_t(15)));
  int2* gidx = reinterpret_cast<int2*>(reinterpret_cast<char*>(goff) + ((size_t(4) * (W + 1) + 15) & ~size_t(15)));
  double* gco = reinterpret_cast<double*>(gidx + T);
  const int4* g_outs = reinterpret_cast<const int4*>(t.sym_outputs);
  const int2* g_gidx = reinterpret_cast<const int2*>(t.sym_grad_index);
  for (int i = threadIdx.x; i < so; i += blockDim.x) outs[i] = __ldg(g_outs + i);
  for (int i = threadIdx.x; i < nterm; i += blockDim.x) {
    fac[i] = __ldg(t.sym_term_factors + i);
    co[i] = __ldg(t.sym_term_coeff + i);
  }
  for (int i = threadIdx.x; i <= W; i += blockDim.x) goff[i] = __ldg(t.sym_grad_offsets + i);
  for (int i = threadIdx.x; i < T; i += blockDim.x) {
    gidx[i] = __ldg(g_gidx + i);
    gco[i] = __ldg(t.sym_grad_coeff + i);
  }
  return SymTabs{outs, fac, co, nterm, goff, gidx, gco};
}

// Symmetric slot: fill values from A.  Threads cover (atom, output) pairs, so
// the two half-warps of a warp fill different outputs (sym_output_tab has no
// data-dependent loop).
__device__ __forceinline__ void grad_fill_slot(const y3b_ace_tables& t, const SymTabs& tb, double2* __restrict__ val,
                                               int W, int slot, int ch) {
  const int na = int(t.nmax) * W, so = int(t.sym_output_count);
  const int atom = threadIdx.x % kGA;
  for (int o = threadIdx.x / kGA; o < so; o += blockDim.x / kGA) {
    const int4 r = tb.outs[o];
    val[(na + slot * so + o) * kGA + atom] =
        sym_output_tab(tb.fac, tb.co, r.y, min(r.z, tb.nterm), val + (ch * W + r.x) * kGA + atom, kGA);
  }
}

// Chain rule from a slot's gradients to the A entries of its radial channel:
// dE/dx_p += sum over monomials containing p of g_o * m * c * prod(other
// factors), from the component-major derivative table.  Each thread owns
// (atom, component) pairs, so the additions need no atomics.
__device__ __forceinline__ void grad_pull_slot(const y3b_ace_tables& t, const SymTabs& tb,
                                               const double2* __restrict__ val, double* __restrict__ Gr,
                                               double* __restrict__ Gi, int W, int slot, int ch) {
  const int na = int(t.nmax) * W, so = int(t.sym_output_count);
  for (int task = threadIdx.x; task < kGA * W; task += blockDim.x) {
    const int atom = task % kGA, comp = task / kGA;
    const double2* x = val + ch * W * kGA + atom;
    const int gb = (na + slot * so) * kGA + atom;
    double ar = 0.0, ai = 0.0;
    const int qe = tb.goff[comp + 1];
    for (int q = tb.goff[comp]; q < qe; ++q) {
      const int2 r = tb.gidx[q];
      const double gr = Gr[gb + r.x * kGA], gi = Gi[gb + r.x * kGA];
      if (gr == 0.0 && gi == 0.0) continue;
      double2 m = make_double2(tb.gco[q], 0.0);
      const uint32_t f = uint32_t(r.y);
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const int ci = (f >> (8 * k)) & 255;
        if (ci != 255) m = mul(m, x[ci * kGA]);
      }
      ar += gr * m.x - gi * m.y;
      ai += gr * m.y + gi * m.x;
    }
    const int e = (ch * W + comp) * kGA + atom;
    Gr[e] += ar;
    Gi[e] += ai;
  }
}

__device__ __forceinline__ void grad_clear_slot(double* __restrict__ Gr, double* __restrict__ Gi, int na, int so,
                                                int slot) {
  for (int e = (na + slot * so) * kGA + threadIdx.x; e < (na + (slot + 1) * so) * kGA; e += blockDim.x)
    Gr[e] = Gi[e] = 0.0;
}

template <int CLS>
__global__ void __launch_bounds__(32 * ClassWarps<CLS>::value, 1) ace_grad_kernel(y3b_ace_tables t, const double2* __restrict__ A,
                                                                   int64_t N, const int32_t* __restrict__ species,
                                                                   const double* __restrict__ weights, int64_t S,
                                                                   double* __restrict__ energy,
                                                                   double2* __restrict__ dEdA,
                                                                   int32_t* __restrict__ status, int accumulate) {
  extern __shared__ double2 gsm[];
  constexpr int kWarps = ClassWarps<CLS>::value;
  __shared__ double red[kWarps][kGA];
  // the run classes (4-block items) read A entries only: no symmetric slots
  constexpr bool kSlots = CLS < kFirstRunClass;
  const int W = int((t.lmax + 1) * (t.lmax + 1));
  const int na = int(t.nmax) * W, so = int(t.sym_output_count);
  const int E = kSlots ? int(t.smem_entries) : na;
  const int rows = E + 2 * kGPad;
  double* Gr = reinterpret_cast<double*>(gsm + rows * kGA);
  double* Gi = Gr + E * kGA;
  double2* stg = reinterpret_cast<double2*>(Gi + E * kGA);
  constexpr int kStageLanes = kSlots ? kStage : kStageRun;  // staged entries per lane
  for (int e = threadIdx.x; e < rows * kGA; e += blockDim.x) gsm[e] = make_double2(0.0, 0.0);
  for (int e = threadIdx.x; e < 2 * E * kGA; e += blockDim.x) Gr[e] = 0.0;
  __syncthreads();
  double2* val = gsm + kGPad * kGA;
  {
    const int la = threadIdx.x % kGA;  // loader thread's atom
    const int64_t aa = blockIdx.x * int64_t(kGA) + la;
    for (int e = threadIdx.x / kGA; e < na; e += blockDim.x / kGA)
      val[e * kGA + la] = aa < N ? A[aa * na + e] : make_double2(0.0, 0.0);
  }
  __syncthreads();  // A is in shared memory before any item reads it
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int atom = lane & (kGA - 1), grp = lane / kGA;
  const int64_t a = blockIdx.x * int64_t(kGA) + atom;
  int z = a < N ? species[a] : 0;
  if (z < 0 || z >= S) {
    if (status && grp == 0) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
    z = 0;
  }
  const double* wz = weights + int64_t(z) * t.feature_count;
  const Ctx c{val + atom, static_cast<uint32_t>(__cvta_generic_to_shared(Gr + atom)),
              static_cast<uint32_t>(__cvta_generic_to_shared(Gi + atom)), stg + warp * kStageLanes * 32 + lane};
  const int4* items = reinterpret_cast<const int4*>(t.items);
  const int4* phases = reinterpret_cast<const int4*>(t.phases);
  const int2* groups = reinterpret_cast<const int2*>(t.groups);
  int cur0 = -2, cur1 = -2;
  double e_acc = 0.0;
  // slot tables staged in the staging area at phase changes when they fit
  const int nterm = kSlots ? sym_term_total(t) : 0;
  const bool tabs_staged =
      kSlots && sym_tabs_bytes(so, nterm, W, t.sym_grad_count) <= size_t(kWarps) * kStageLanes * 32 * sizeof(double2);
  const SymTabs tg = sym_tabs_global(t, nterm);
  if (!kSlots) {
    // four-block classes: all pairs sit in phase 0's range (no slots), one
    // contiguous run per warp
    const int gb = __ldg(t.group_offsets + CLS * (t.phase_count + 1));
    const int ge = __ldg(t.group_offsets + CLS * (t.phase_count + 1) + 1);
    const int per = (ge - gb + kWarps - 1) / kWarps;
    const int g0 = gb + warp * per, g1 = min(ge, g0 + per);
    bool bad = false;
    e_acc = adj4_run<CLS>(c, groups, g0, g1, grp, items, t.item_coef, wz, bad);
    if (bad && status) atomicOr(status, Y3B_STATUS_TABLE);
  }
#pragma unroll 1
  for (int ph = 0; kSlots && ph < t.phase_count; ++ph) {
    const int4 pr = __ldg(phases + ph);
    const int* goff = t.group_offsets + CLS * (t.phase_count + 1);
    const int gb = __ldg(goff + ph), ge = __ldg(goff + ph + 1);
    if (gb == ge) continue;  // no items of this class in the phase
    if (kSlots && (pr.x != cur0 || pr.y != cur1)) {
      __syncthreads();  // the previous phase is done with the slots and the staging area
      const SymTabs tb = tabs_staged ? sym_tabs_stage(t, reinterpret_cast<char*>(stg), nterm, W) : tg;
      if (tabs_staged) __syncthreads();
      if (pr.x != cur0 && cur0 >= 0) grad_pull_slot(t, tb, val, Gr, Gi, W, 0, cur0);
      if (pr.y != cur1 && cur1 >= 0) grad_pull_slot(t, tb, val, Gr, Gi, W, 1, cur1);
      __syncthreads();
      if (pr.x != cur0) {
        grad_clear_slot(Gr, Gi, na, so, 0);
        grad_fill_slot(t, tb, val, W, 0, pr.x);
      }
      if (pr.y != cur1) {
        if (t.smem_entries >= na + 2 * so) grad_clear_slot(Gr, Gi, na, so, 1);
        if (pr.y >= 0 && t.smem_entries >= na + 2 * so) grad_fill_slot(t, tb, val, W, 1, pr.y);
      }
      __syncthreads();
      cur0 = pr.x;
      cur1 = pr.y;
    }
    if constexpr (CLS == 1) {
      // one sorted run per warp (packing pads the phase's range to equal runs)
      const int per = (ge - gb + kWarps - 1) / kWarps;
      const int g0 = gb + warp * per, g1 = min(ge, g0 + per);
      bool bad = false;
      e_acc += adj3_run(c, groups, g0, g1, grp, items, t.item_coef, wz, bad);
      if (bad && status) atomicOr(status, Y3B_STATUS_TABLE);
    } else {
#pragma unroll 1
      for (int g = gb + warp; g < ge; g += kWarps) {
        const int2 ig = __ldg(groups + g);
        if (ig.x < 0) continue;  // null pair
        const int mine = grp == 0 ? ig.x : ig.y;
        const bool mute = mine < 0;  // odd item out: the second half runs the first item unweighted, adding nothing
        const Item it = load_item(items, mute ? ig.x : mine);
        const double w0 = mute ? 0.0 : __ldg(wz + it.f0);
        const double w1 = (!mute && it.f1 >= 0) ? __ldg(wz + it.f1) : 0.0;
        e_acc += adj_class<0>(c, it, t.item_coef, w0, w1, mute);
      }
    }
  }
  __syncthreads();
  if (kSlots && (cur0 >= 0 || cur1 >= 0)) {
    const SymTabs tb = tabs_staged ? sym_tabs_stage(t, reinterpret_cast<char*>(stg), nterm, W) : tg;
    if (tabs_staged) __syncthreads();
    if (cur0 >= 0) grad_pull_slot(t, tb, val, Gr, Gi, W, 0, cur0);
    if (cur1 >= 0) grad_pull_slot(t, tb, val, Gr, Gi, W, 1, cur1);
  }
  e_acc += __shfl_xor_sync(0xffffffffu, e_acc, 16);
  if (grp == 0) red[warp][atom] = e_acc;
  __syncthreads();
  if (threadIdx.x < kGA) {
    const int64_t aa = blockIdx.x * int64_t(kGA) + threadIdx.x;
    double s = 0.0;
    for (int w = 0; w < kWarps; ++w) s += red[w][threadIdx.x];
    if (aa < N) energy[aa] = accumulate ? energy[aa] + s : s;
  }
  {
    const int la = threadIdx.x % kGA;
    const int64_t aa = blockIdx.x * int64_t(kGA) + la;
    for (int e = threadIdx.x / kGA; e < na; e += blockDim.x / kGA)
      if (aa < N) {
        double2 g = make_double2(Gr[e * kGA + la], Gi[e * kGA + la]);
        if (accumulate) g = add(g, dEdA[aa * na + e]);
        dEdA[aa * na + e] = g;
      }
  }
}

// ---------------------------------------------------------------------------
// Edge gradients: one warp per centre i; lanes over its edges.  With
// A[n, lm] = sum_j p_j R_n(r) Yc_lm(d),  g_e = dE_i/dd_e =
//   p_j ( d_hat sum_lm Re(Q_lm Yc_lm) + sum_lm Re(P_lm grad Yc_lm) ),
//   P_lm = sum_n R_n G[n, lm],  Q_lm = sum_n R'_n G[n, lm].
// The radial table is instantiated at NMAXT >= nmax entries (G is zero
// beyond nmax in shared memory), so radial values and derivatives stay in
// registers; P and Q are formed per harmonic column and used at once.
// ---------------------------------------------------------------------------
constexpr int kEdgeWarps = 4;

// CTAs per SM the register allocation aims at: 4 (at most 128 registers) for l_max <= 3
// with an 8-entry radial table, 11 % faster than 3 there; 3 for the larger instances
template <int LMAX, int NMAXT>
struct EdgeMinBlocks {
  static constexpr int value = (LMAX <= 3 && NMAXT <= 8) ? 4 : 3;
};

template <int LMAX, int NMAXT>
__global__ void __launch_bounds__(32 * kEdgeWarps, EdgeMinBlocks<LMAX, NMAXT>::value) ace_edge_grad_kernel(
    const double* __restrict__ pos, const int32_t* __restrict__ species, int64_t N, int64_t center_begin,
    int64_t count, double box, const int64_t* __restrict__ row_off, const int32_t* __restrict__ nbr,
    const double* __restrict__ pref, int64_t S, int nmax, double rc, double lam, ShNorm nrm,
    const double2* __restrict__ dEdA, double* __restrict__ edge_grad, int32_t* status) {
  constexpr int W = (LMAX + 1) * (LMAX + 1);
  // dE/dA of the centre folded into the real-harmonic basis: with Yc_lm = sum_k
  // T[lm, k] Y_k (Yc_{l,0} = Y_{l,0}; Yc_{l,-m} = (Y_{l,m} + i Y_{l,-m}) / sqrt 2;
  // Yc_{l,m} = (-1)^m (Y_{l,m} - i Y_{l,-m}) / sqrt 2), sum_lm Re(G[n, lm] Yc_lm) =
  // sum_k Gr[n, k] Y_k with Gr[n, k] = Re(sum_lm G[n, lm] T[lm, k]), so every edge
  // contracts real channels (half the multiply-adds of the complex form)
  __shared__ double sG[kEdgeWarps][NMAXT * W];
  __shared__ double2 sGc[kEdgeWarps][NMAXT * W];  // the centre's dE/dA row as read
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int na = nmax * W;
  const int64_t row0 = row_off[0];
  const double inv2 = 0.70710678118654752440084436210484903;
  for (int64_t c = blockIdx.x * int64_t(kEdgeWarps) + wib; c < count; c += int64_t(gridDim.x) * kEdgeWarps) {
    const int64_t i = center_begin + c;
    for (int q = lane; q < NMAXT * W; q += 32) sGc[wib][q] = q < na ? dEdA[c * na + q] : make_double2(0.0, 0.0);
    __syncwarp();
    for (int q = lane; q < NMAXT * W; q += 32) {
      const int n = q / W, k = q - n * W;
      const int l = int(sqrtf(float(k)));
      const int cc = l * l + l, m = k - cc, am = m < 0 ? -m : m;
      const double2* Gn = sGc[wib] + n * W;
      double gr;
      if (m == 0) {
        gr = Gn[cc].x;
      } else {
        const double sg = (am & 1) ? -1.0 : 1.0;
        const double2 gm = Gn[cc - am], gp = Gn[cc + am];
        gr = m > 0 ? inv2 * (gm.x + sg * gp.x) : inv2 * (sg * gp.y - gm.y);
      }
      sG[wib][q] = gr;
    }
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
        double rv[NMAXT + 1], rd[NMAXT + 1];
        radial_basis<double>(r, rc, lam, NMAXT, rv, rd);
        const double eps = 1e-12;
        const double sr = r > eps ? r : eps;
        const double u[3] = {d[0] / sr, d[1] / sr, d[2] / sr};
        ShState<double, LMAX> st;
        sh_state<double, LMAX>(u[0], u[1], u[2], st);
        // Cartesian gradients of the real harmonics: J = (I - u u^T) / |d| (I / eps
        // below eps), as ye3t_runtime_core.cpp:819-834; the division by |d| is one
        // reciprocal and a product per entry
        const double inv_sr = 1.0 / sr;
        double acc_r = 0.0, acc_v[3] = {0.0, 0.0, 0.0};
        // one real harmonic k with its gradient: add Q_k Y_k and P_k grad Y_k with
        // P_k = sum_n R_n Gr[n, k], Q_k = sum_n R'_n Gr[n, k]
        auto column = [&](int k, double y, const double (&dy)[3]) {
          double P = 0.0, Q = 0.0;
#pragma unroll
          for (int n = 0; n < NMAXT; ++n) {
            const double gv = sG[wib][n * W + k];
            P = fma(rv[n + 1], gv, P);
            Q = fma(rd[n + 1], gv, Q);
          }
          acc_r = fma(Q, y, acc_r);
#pragma unroll
          for (int ax = 0; ax < 3; ++ax) acc_v[ax] = fma(P, dy[ax], acc_v[ax]);
        };
#pragma unroll
        for (int l = 0; l <= LMAX; ++l) {
          const int cidx = l * l + l;
#pragma unroll
          for (int m = 0; m <= l; ++m) {
            double v[2], g[2][3];
            real_sh_pair<double, LMAX>(l, m, st, nrm, v, g);
#pragma unroll
            for (int h = 0; h < (m == 0 ? 1 : 2); ++h) {
              const double gu = r > eps ? g[h][0] * u[0] + g[h][1] * u[1] + g[h][2] * u[2] : 0.0;
#pragma unroll
              for (int ax = 0; ax < 3; ++ax) g[h][ax] = (g[h][ax] - gu * u[ax]) * inv_sr;
            }
            column(cidx + m, v[0], g[0]);
            if (m > 0) column(cidx - m, v[1], g[1]);
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
  Y3B_CHECK_ARG(t->group_offsets && (t->group_count == 0 || t->groups), "null adjoint item groups");
  Y3B_CHECK_ARG(t->sym_grad_offsets && (t->sym_grad_count == 0 || (t->sym_grad_index && t->sym_grad_coeff)),
                "null symmetric derivative tables");
  Y3B_CHECK_ARG(t->sym_term_count >= 0 && (t->sym_output_count == 0 || t->sym_term_count > 0),
                "symmetric term count missing");
  return Y3B_OK;
}

}  // namespace
}  // namespace y3b

using namespace y3b;

extern "C" int y3b_ace_energy_grad(const y3b_ace_tables* tables, const void* A, int64_t atom_count,
                                   const int32_t* species, const double* weights, int64_t species_count,
                                   double* energy, void* dEdA, int32_t* status, void* stream) {
  if (int rc = check_grad_tables(tables)) return rc;
  Y3B_CHECK_ARG(atom_count >= 0, "negative atom count");
  if (atom_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(A && species && weights && energy && dEdA && species_count > 0, "null pointer argument");
  auto smem_for = [&](int64_t entries, int stage, int warps) {
    return size_t(entries + 2 * kGPad) * kGA * sizeof(double2) + size_t(2) * size_t(entries) * kGA * sizeof(double) +
           size_t(warps) * stage * 32 * sizeof(double2);
  };
  const size_t smem = smem_for(tables->smem_entries, kStage, kGWarps);
  const size_t smem_a = smem_for(tables->nmax * (tables->lmax + 1) * (tables->lmax + 1), kStageRun, kGWarpsRun);
  Y3B_CHECK_ARG(smem_a <= 224 * 1024, "adjoint run path needs %lld bytes of shared memory (max 224 KB)",
                (long long)smem_a);
  Y3B_CHECK_ARG(smem <= 224 * 1024, "bundle needs %lld bytes of shared memory for the adjoint (max 224 KB)",
                (long long)smem);
  const int64_t grid = (atom_count + kGA - 1) / kGA;
  Y3B_CHECK_ARG(grid < (int64_t(1) << 31), "too many atoms");
  cudaStream_t s = as_stream(stream);
  // one launch per item class (stream-ordered); the first writes dE/dA and
  // the energies, the others add to them
#define Y3B_GRAD_LAUNCH(CLS)                                                                              \
  Y3B_CUDA_TRY(cudaFuncSetAttribute(ace_grad_kernel<CLS>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                    int(CLS < kFirstRunClass ? smem : smem_a)));                          \
  ace_grad_kernel<CLS><<<int(grid), 32 * ClassWarps<CLS>::value, CLS < kFirstRunClass ? smem : smem_a, s>>>( \
      *tables, static_cast<const double2*>(A),                                                            \
                                                             atom_count, species, weights, species_count, \
                                                             energy, static_cast<double2*>(dEdA), status, \
                                                             CLS > 0);                                    \
  Y3B_LAUNCH_CHECK();
  Y3B_GRAD_LAUNCH(0)
  Y3B_GRAD_LAUNCH(1)
  Y3B_GRAD_LAUNCH(2)
  Y3B_GRAD_LAUNCH(3)
#undef Y3B_GRAD_LAUNCH
  static_assert(kGradClasses == 4, "one launch per class");
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
#define Y3B_EDGE_LAUNCH(L, NT)                                                                              \
  ace_edge_grad_kernel<L, NT><<<grid, 32 * kEdgeWarps, 0, s>>>(                                             \
      positions, species, atom_count, center_begin, center_count, box, row_offsets, neighbors,              \
      species_prefactor, species_count, int(nmax), cutoff, lambda, nrm, static_cast<const double2*>(dEdA),   \
      edge_grad, status)
#define Y3B_EDGE_CASE(L)                                                                                    \
  case L:                                                                                                   \
    if (nmax <= 8) Y3B_EDGE_LAUNCH(L, 8);                                                                   \
    else if (nmax <= 12) Y3B_EDGE_LAUNCH(L, 12);                                                            \
    else Y3B_EDGE_LAUNCH(L, 16);                                                                            \
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
#undef Y3B_EDGE_LAUNCH
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
