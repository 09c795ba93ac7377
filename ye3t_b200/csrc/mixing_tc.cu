// Mixed-channel A-basis on the tensor cores (fp32).
//
// The per-species-pair radial mixing of y3b_ace_density_mixed,
//   A[i, c, lm] = sum_{j in row i} sum_n W[z_i, z_j, c, n] R_n(r_ij) Yc_lm(r_ij),
// is regrouped so that the mixing becomes one matrix product per 128 rows:
//   S[i, lm, z, n] = sum_{j in row i, z_j = z} R_n(r_ij) Yc_lm(r_ij)        (CUDA cores)
//   A[i, c, lm]    = sum_{z, n} W[z_i, z, c, n] S[i, lm, z, n]              (tcgen05)
// The first kernel is the A-basis of ye3t/runtime/execution_plan.py:7298 (radial
// table), :7479 (complex harmonics) and :7913 (density_accumulate) with the sum split
// by neighbour species; the second applies pace_radial_channel_contraction
// (ye3t/runtime/csrc/ye3t_runtime_core.cpp:651) to the summed rows.
//
// The product: rows (atom, lm, real/imaginary part) of S, K = (z, n) padded to a
// multiple of 8, and N = (centre species s, channel c): every centre species' table
// is applied to every row and the epilogue keeps the block of the row's own species,
// so that a tile of 128 rows needs no sorting by species.  It runs as
// tcgen05.mma kind::tf32 with fp32 accumulators in tensor memory, each operand
// split into a TF32 high part and the TF32 rounding of the remainder (3xTF32:
// hi*hi + hi*lo + lo*hi), which keeps the error near fp32 rounding.
#include "common.cuh"
#include "edge_math.cuh"
#include "neighbors.cuh"

namespace y3b {

namespace {

constexpr int kTcMaxRadial = 16;
constexpr int kSpWarps = 4;
constexpr int kTcRows = 128;          // M of one tcgen05.mma (rows per tile)
constexpr int kTcThreads = 128;       // one thread per row of the tile
constexpr int kTcMaxK = 64;           // S * nmax padded to 8
constexpr int kTcMaxN = 256;          // S * C padded to 16
constexpr int kWaitLimit = 1 << 22;   // polls of an mbarrier before the kernel gives up

// ---------------------------------------------------------------------------
// Species-split densities S: one warp per centre.  Pass 1: lanes over up to 32
// edges form R_n and the real harmonics Y_k in warp-private shared memory (each
// lane keeps its edge's species).  Pass 2: lane (k, g) owns real harmonic k and every
// G-th radial index, G = 32 / (lmax+1)^2, and for each species sums the chunk's
// edges of that species (a warp ballot) in CSR order into the centre's real-basis rows, kept in
// shared memory across the chunks of rows longer than 32 edges.  The complex
// harmonics are fixed combinations of the real ones (Yc_{l,0} = Y_{l,0};
// Yc_{l,-m} = (Y_{l,m} + i Y_{l,-m}) / sqrt 2; Yc_{l,m} = (-1)^m (Y_{l,m} -
// i Y_{l,-m}) / sqrt 2), so the complex rows (a, lm, part) of Kp values (column
// z * nmax + n, zero padded) are formed from the summed real rows as they are
// written out, consecutive lanes on consecutive values.
template <typename T, int LMAX>
__global__ void __launch_bounds__(32 * kSpWarps) ace_species_density_kernel(
    const double* __restrict__ pos, const int32_t* __restrict__ species, int64_t N, int64_t center_begin,
    int64_t a_begin, int64_t a_count, double box, const int64_t* __restrict__ row_off,
    const int32_t* __restrict__ nbr, int S, int nmax, int Kp, T rc, T lam, ShNorm nrm,
    T* __restrict__ Sout, int32_t* status) {
  constexpr int W = (LMAX + 1) * (LMAX + 1);
  constexpr int W2 = 2 * W;
  constexpr int G = 32 / W;
  constexpr int NPL = (kTcMaxRadial + G - 1) / G;  // radial indices per lane
  constexpr int RS = kTcMaxRadial + 4;             // radial row (16-byte multiple)
  __shared__ __align__(16) T s_r[kSpWarps][32 * RS];
  __shared__ T s_y[kSpWarps][32 * W];
  extern __shared__ __align__(16) unsigned char sp_dyn[];
  T* s_rows = reinterpret_cast<T*>(sp_dyn);  // [warp][W][Kp + 1], real basis
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  T* r_w = s_r[wib];
  T* y_w = s_y[wib];
  const int KS = Kp + 1;
  T* o_w = s_rows + wib * W * KS;
  const int k = lane % W, g = lane / W;
  const bool owner = lane < G * W;
  const int64_t row0 = row_off[0];
  const T inv2 = T(0.70710678118654752440084436210484903);
  for (int64_t al = blockIdx.x * int64_t(kSpWarps) + wib; al < a_count; al += int64_t(gridDim.x) * kSpWarps) {
    const int64_t a = a_begin + al;  // index within the centre range
    const int64_t i = center_begin + a;
    const int64_t b = row_off[a] - row0, e = row_off[a + 1] - row0;
    for (int u = lane; u < W * KS; u += 32) o_w[u] = T(0);
    __syncwarp();
    for (int64_t c0 = b; c0 < e; c0 += 32) {
      const int nedge = (e - c0) < 32 ? int(e - c0) : 32;
      int my_z = -1;  // the species of this lane's edge (-1: none or out of range)
      if (lane < nedge) {
        const int64_t j = nbr[c0 + lane];
        const int zj = (j >= 0 && j < N) ? species[j] : -1;
        if (j < 0 || j >= N || zj < 0 || zj >= S) {
          if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
        } else {
          my_z = zj;
          double dd[3];
          min_image(pos, i, j, box, dd);
          const double r2 = dist2(dd);
          const T d[3] = {T(dd[0]), T(dd[1]), T(dd[2])};
          const T r = sqrt(T(r2));
          T rv[kTcMaxRadial + 1];
          radial_basis<T>(r, rc, lam, nmax, rv, nullptr);
          for (int n = 0; n < nmax; ++n) r_w[lane * RS + n] = rv[n + 1];
          const T sr = r > T(1e-12) ? r : T(1e-12);
          T v[W];
          real_sh_unit<T, LMAX>(d[0] / sr, d[1] / sr, d[2] / sr, nrm, v, nullptr);
#pragma unroll
          for (int q = 0; q < W; ++q) y_w[lane * W + q] = v[q];
        }
      }
      __syncwarp();
      for (int z = 0; z < S; ++z) {
        T acc[NPL];
#pragma unroll
        for (int t = 0; t < NPL; ++t) acc[t] = T(0);
        // the chunk's edges of species z, in CSR order (the same mask in every lane)
        for (unsigned m = __ballot_sync(0xffffffffu, my_z == z); m != 0u; m &= m - 1u) {
          const int q = __ffs(int(m)) - 1;
          const T y = y_w[q * W + k];
          const T* rq = r_w + q * RS;
          if constexpr (G == 1 && sizeof(T) == 4) {
#pragma unroll
            for (int t = 0; t < NPL; t += 4) {
              if (t < nmax) {
                const float4 r4 = *reinterpret_cast<const float4*>(rq + t);
                acc[t] = fma(T(r4.x), y, acc[t]);
                acc[t + 1] = fma(T(r4.y), y, acc[t + 1]);
                acc[t + 2] = fma(T(r4.z), y, acc[t + 2]);
                acc[t + 3] = fma(T(r4.w), y, acc[t + 3]);
              }
            }
          } else {
#pragma unroll
            for (int t = 0; t < NPL; ++t) {
              const int n = g + t * G;
              if (n < nmax) acc[t] = fma(rq[n], y, acc[t]);
            }
          }
        }
        if (owner) {
#pragma unroll
          for (int t = 0; t < NPL; ++t) {
            const int n = g + t * G;
            if (n < nmax) o_w[k * KS + z * nmax + n] += acc[t];
          }
        }
      }
      __syncwarp();
    }
    T* So = Sout + al * int64_t(W2) * Kp;
    for (int u = lane; u < W2 * Kp; u += 32) {
      const int row = u / Kp, col = u - row * Kp;
      const int lm = row >> 1, part = row & 1;
      int l = 0;
      while ((l + 1) * (l + 1) <= lm) ++l;
      const int m = lm - l * l - l, cc = l * l + l, am = m < 0 ? -m : m;
      T val;
      if (m == 0) {
        val = part ? T(0) : o_w[cc * KS + col];
      } else {
        const T sg = (m > 0 && (am & 1)) ? T(-1) : T(1);
        // m < 0: (Y_{l,|m|} + i Y_{l,-|m|}) / sqrt 2; m > 0: (-1)^m (Y_{l,m} - i Y_{l,-m}) / sqrt 2
        val = part ? (m < 0 ? T(1) : T(-1)) * sg * inv2 * o_w[(cc - am) * KS + col]
                   : sg * inv2 * o_w[(cc + am) * KS + col];
      }
      So[u] = val;
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// tcgen05 helpers (inline PTX, sm_100a).

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Shared-memory matrix descriptor, no swizzle, K-major: core matrices of 8 rows x
// 16 bytes, rows 16 bytes apart; lbo = bytes between the two 16-byte K halves of one
// MMA's K = 8, sbo = bytes between 8-row groups; version 1 (bits 46-47).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}

// Instruction descriptor of kind::tf32: fp32 accumulator (bits 4-5 = 1), A and B
// TF32 (bits 7-9, 10-12 = 2), both K-major, N >> 3 at bits 17-22, M >> 4 at 24-28.
__device__ __forceinline__ uint32_t tf32_idesc(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(mbar)
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t mbar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(mbar), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

// ---------------------------------------------------------------------------
// Mixing product on the tensor cores.  A persistent CTA of 128 threads: thread t
// loads row t of a tile of S, splits it into TF32 hi/lo parts in the no-swizzle
// K-major layout (16-byte K chunk kc of row t at (kc * 128 + t) * 16 bytes);
// thread 0 issues 3 MMAs per K step of 8 into the tile's accumulator in tensor
// memory and commits them to an mbarrier; after the wait every warp reads its 32
// rows (tensor-memory lanes 32w..32w+31) 16 columns at a time and writes the
// columns of the row's centre species into A.  The B operand (every centre
// species' table, rows (s, c), K = (z, n)) is split and staged once per CTA.
// A wait that runs out sets Y3B_STATUS_TIMEOUT and ends the CTA's loop.
__global__ void __launch_bounds__(kTcThreads) mixing_tf32_kernel(
    const float* __restrict__ Sin, int64_t atom_count, int W2, int Kp, const float* __restrict__ mix, int S, int C,
    int nmax, int Np, int tmem_cols, const int32_t* __restrict__ species, float* __restrict__ A, int32_t* status) {
  extern __shared__ __align__(1024) unsigned char tc_smem[];
  __shared__ uint64_t mbar;
  __shared__ uint32_t tmem_base_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  float* sAhi = reinterpret_cast<float*>(tc_smem);
  float* sAlo = sAhi + kTcRows * Kp;
  float* sBhi = sAlo + kTcRows * Kp;
  float* sBlo = sBhi + Np * Kp;
  const uint32_t mbar_a = smem_u32(&mbar);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(mbar_a) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  // B operand: row (s, c) of Np, column (z, n) of Kp; zero outside S * C x S * nmax
  for (int u = tid; u < Np * Kp; u += kTcThreads) {
    const int nr = u / Kp, k = u - nr * Kp;
    float v = 0.0f;
    if (nr < S * C && k < S * nmax) {
      const int s = nr / C, c = nr - s * C, z = k / nmax, n = k - z * nmax;
      v = mix[((int64_t(s) * S + z) * C + c) * nmax + n];
    }
    const float hi = tf32_round(v);
    const int off = ((k >> 2) * Np + nr) * 4 + (k & 3);
    sBhi[off] = hi;
    sBlo[off] = tf32_round(v - hi);
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = tmem_base_s;
  const uint32_t idesc = tf32_idesc(kTcRows, Np);
  const int64_t rows = atom_count * W2;
  const int64_t tiles = (rows + kTcRows - 1) / kTcRows;
  const int ksteps = Kp / 8;
  uint32_t parity = 0;
  // the rows of the CTA's next tile, loaded while the current tile's MMAs run
  float4 nxt[kTcMaxK / 4];
  auto fetch = [&](int64_t tile) {
    const int64_t r = tile * kTcRows + tid;
    const bool ok = tile < tiles && r < rows;
    const float4* src = reinterpret_cast<const float4*>(Sin + (ok ? r : 0) * Kp);
#pragma unroll
    for (int kc = 0; kc < kTcMaxK / 4; ++kc)
      if (kc < Kp / 4) nxt[kc] = ok ? src[kc] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  };
  fetch(blockIdx.x);
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t r = tile * kTcRows + tid;
    const bool valid = r < rows;
#pragma unroll
    for (int kc = 0; kc < kTcMaxK / 4; ++kc) {
      if (kc < Kp / 4) {
        const float4 v = nxt[kc];
        float4 hi, lo;
        hi.x = tf32_round(v.x);
        hi.y = tf32_round(v.y);
        hi.z = tf32_round(v.z);
        hi.w = tf32_round(v.w);
        lo.x = tf32_round(v.x - hi.x);
        lo.y = tf32_round(v.y - hi.y);
        lo.z = tf32_round(v.z - hi.z);
        lo.w = tf32_round(v.w - hi.w);
        reinterpret_cast<float4*>(sAhi)[kc * kTcRows + tid] = hi;
        reinterpret_cast<float4*>(sAlo)[kc * kTcRows + tid] = lo;
      }
    }
    // generic-proxy writes of the operands become visible to the tensor cores
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      const uint32_t a_hi = smem_u32(sAhi), a_lo = smem_u32(sAlo), b_hi = smem_u32(sBhi), b_lo = smem_u32(sBlo);
      const uint32_t a_lbo = kTcRows * 16, b_lbo = uint32_t(Np) * 16;
      for (int ks = 0; ks < ksteps; ++ks) {
        const uint32_t ao = uint32_t(ks) * 2 * a_lbo, bo = uint32_t(ks) * 2 * b_lbo;
        mma_tf32(tmem, smem_desc(a_lo + ao, a_lbo, 128), smem_desc(b_hi + bo, b_lbo, 128), idesc, ks > 0);
        mma_tf32(tmem, smem_desc(a_hi + ao, a_lbo, 128), smem_desc(b_lo + bo, b_lbo, 128), idesc, 1);
        mma_tf32(tmem, smem_desc(a_hi + ao, a_lbo, 128), smem_desc(b_hi + bo, b_lbo, 128), idesc, 1);
      }
      mma_commit(mbar_a);
    }
    fetch(tile + gridDim.x);
    bool done = false;
    for (int it = 0; it < kWaitLimit && !done; ++it) done = mbar_test(mbar_a, parity);
    if (__syncthreads_or(!done)) {
      if (tid == 0 && status) atomicOr(status, Y3B_STATUS_TIMEOUT);
      break;
    }
    parity ^= 1u;
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const int64_t a = valid ? r / W2 : 0;
    const int rem = int(r - a * W2);
    int zi = valid ? species[a] : -1;
    if (valid && (zi < 0 || zi >= S)) {
      if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
      zi = -1;
    }
    float* Ao = A + a * int64_t(C) * W2 + rem;
    const uint32_t lane_base = tmem + (uint32_t(32 * warp) << 16);
    for (int s = 0; s < S; ++s) {
      for (int c0 = 0; c0 < C; c0 += 16) {
        float v[16];
        tmem_ld16(lane_base + uint32_t(s * C + c0), v);
        if (valid && zi == s) {
#pragma unroll
          for (int j = 0; j < 16; ++j) Ao[int64_t(c0 + j) * W2] = v[j];
        }
      }
    }
    if (valid && zi < 0)
      for (int c = 0; c < C; ++c) Ao[int64_t(c) * W2] = 0.0f;
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  }
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(tmem_cols) : "memory");
}

// ---------------------------------------------------------------------------
// Mixing product in fp64 on the FP64 tensor cores (mma.sync m8n8k4; tcgen05 has
// no FP64 kind).  A warp takes 8 rows (a, lm, part) of one centre (a centre's rows
// padded to a multiple of 8) and the C channels of the centre's species: per K step
// of 4, the A fragment S[row l/4][4 ks + l%4] (global memory, through L1) and for
// each block of 8 channels the B fragment W[z_i][k][c] from shared memory (rows of
// C + 8 doubles, so that the four k rows of a fragment fall in two halves of the
// banks); lane l ends with D[row l/4][c = 8 nb + 2 (l%4) + {0, 1}].
constexpr int kF64Warps = 8;
constexpr int kF64MaxNB = 8;  // C <= 64

__device__ __forceinline__ void dmma_f64(double& d0, double& d1, double a, double b) {
  asm("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};\n"
      : "+d"(d0), "+d"(d1)
      : "d"(a), "d"(b));
}

__global__ void __launch_bounds__(32 * kF64Warps) mixing_f64_kernel(
    const double* __restrict__ Sin, int64_t atom_count, int W2, int Kp, const double* __restrict__ mix, int S, int C,
    int nmax, const int32_t* __restrict__ species, double* __restrict__ A, int32_t* status) {
  extern __shared__ __align__(16) unsigned char f64_smem[];
  double* sW = reinterpret_cast<double*>(f64_smem);  // [s][k][C + 8]
  const int CS = C + 8;
  for (int u = threadIdx.x; u < S * Kp * C; u += blockDim.x) {
    const int sz = u / (Kp * C), rem = u - sz * Kp * C, k = rem / C, c = rem - k * C;
    double v = 0.0;
    if (k < S * nmax) {
      const int z = k / nmax, n = k - z * nmax;
      v = mix[((int64_t(sz) * S + z) * C + c) * nmax + n];
    }
    sW[(sz * Kp + k) * CS + c] = v;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int kk = lane & 3, r = lane >> 2;
  const int RB = (W2 + 7) / 8;  // row blocks per centre
  const int64_t tasks = atom_count * RB;
  const int nbs = C / 8;
  for (int64_t task = blockIdx.x * int64_t(kF64Warps) + warp; task < tasks;
       task += int64_t(gridDim.x) * kF64Warps) {
    const int64_t a = task / RB;
    const int rb = int(task - a * RB);
    int zi = species[a];
    const bool zok = zi >= 0 && zi < S;
    if (!zok) {
      if (status && lane == 0 && rb == 0) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
      zi = 0;
    }
    const int row = rb * 8 + r;
    const bool rok = row < W2;
    const double* Srow = Sin + (a * W2 + (rok ? row : 0)) * Kp + kk;
    const double* Wz = sW + (int64_t(zi) * Kp + kk) * CS + r;  // B[k = 4 ks + kk][c = 8 nb + r]
    double acc[kF64MaxNB][2];
#pragma unroll
    for (int nb = 0; nb < kF64MaxNB; ++nb) acc[nb][0] = acc[nb][1] = 0.0;
    // the lane's A fragments of every K step, loaded together ahead of the products
    double av[kTcMaxK / 4];
#pragma unroll
    for (int ks = 0; ks < kTcMaxK / 4; ++ks) av[ks] = (rok && ks < Kp / 4) ? Srow[4 * ks] : 0.0;
#pragma unroll
    for (int ks = 0; ks < kTcMaxK / 4; ++ks) {
      if (ks >= Kp / 4) break;  // uniform over the warp
      const double* Wk = Wz + 4 * ks * CS;
#pragma unroll
      for (int nb = 0; nb < kF64MaxNB; ++nb)
        if (nb < nbs) dmma_f64(acc[nb][0], acc[nb][1], av[ks], Wk[8 * nb]);  // uniform over the warp
    }
    if (rok) {
      double* Ao = A + a * int64_t(C) * W2 + row;
#pragma unroll
      for (int nb = 0; nb < kF64MaxNB; ++nb) {
        if (nb < nbs) {
          const int c = 8 * nb + 2 * kk;
          Ao[int64_t(c) * W2] = zok ? acc[nb][0] : 0.0;
          Ao[int64_t(c + 1) * W2] = zok ? acc[nb][1] : 0.0;
        }
      }
    }
  }
}

int tc_dims(int64_t S, int64_t C, int64_t nmax, int64_t lmax, int& Kp, int& Np, int& cols) {
  Kp = int((S * nmax + 7) / 8 * 8);
  Np = int((S * C + 15) / 16 * 16);
  cols = 32;
  while (cols < Np) cols *= 2;
  if (lmax < 0 || lmax > 4 || nmax < 1 || nmax > kTcMaxRadial || S < 1 || C < 16 || C % 16 || Kp > kTcMaxK ||
      Np > kTcMaxN)
    return -1;
  return 0;
}

}  // namespace
}  // namespace y3b

using namespace y3b;

namespace y3b {
namespace {

int f64_dims(int64_t S, int64_t C, int64_t nmax, int64_t lmax, int& Kp) {
  Kp = int((S * nmax + 3) / 4 * 4);
  if (lmax < 0 || lmax > 4 || nmax < 1 || nmax > kTcMaxRadial || S < 1 || C < 8 || C % 8 || C > 8 * kF64MaxNB ||
      Kp > kTcMaxK ||
      size_t(S) * Kp * (C + 8) * sizeof(double) > 200 * 1024)
    return -1;
  return 0;
}

int split_dims(int dtype, int64_t S, int64_t C, int64_t nmax, int64_t lmax, int& Kp, int& Np, int& cols) {
  Np = cols = 0;
  if (dtype == Y3B_F32) return tc_dims(S, C, nmax, lmax, Kp, Np, cols);
  if (dtype == Y3B_F64) return f64_dims(S, C, nmax, lmax, Kp);
  return -1;
}

}  // namespace
}  // namespace y3b

extern "C" int64_t y3b_ace_density_mixed_split_workspace_bytes(int dtype, int64_t center_count,
                                                               int64_t species_count, int64_t channel_count,
                                                               int64_t nmax, int64_t lmax) {
  int Kp = 0, Np = 0, cols = 0;
  if (center_count < 0 || split_dims(dtype, species_count, channel_count, nmax, lmax, Kp, Np, cols)) return -1;
  const int64_t real = dtype == Y3B_F64 ? 8 : 4;
  return center_count * 2 * (lmax + 1) * (lmax + 1) * Kp * real;
}

extern "C" int y3b_ace_density_mixed_split(int dtype, const double* positions, const int32_t* species,
                                           int64_t atom_count, int64_t center_begin, int64_t center_count,
                                           double box, const int64_t* row_offsets, const int32_t* neighbors,
                                           const void* mixing, int64_t species_count, int64_t channel_count,
                                           int64_t nmax, int64_t lmax, double cutoff, double lambda,
                                           void* workspace, int64_t workspace_bytes, void* A, int32_t* status,
                                           void* stream) {
  int Kp = 0, Np = 0, cols = 0;
  Y3B_CHECK_ARG(dtype == Y3B_F32 || dtype == Y3B_F64, "ace_density_mixed_split: dtype must be F32 or F64");
  if (split_dims(dtype, species_count, channel_count, nmax, lmax, Kp, Np, cols))
    return fail(Y3B_ERR_UNSUPPORTED,
                dtype == Y3B_F32
                    ? "ace_density_mixed_split (fp32, tcgen05): needs lmax <= 4, nmax <= 16, C a multiple of 16, "
                      "S * nmax <= 64 and S * C <= 256"
                    : "ace_density_mixed_split (fp64): needs lmax <= 4, nmax <= 16, C a multiple of 8 up to 64 "
                      "and S * Kp * (C + 8) doubles within 200 KB");
  Y3B_CHECK_ARG(center_begin >= 0 && center_count >= 0 && center_begin + center_count <= atom_count,
                "bad centre range");
  Y3B_CHECK_ARG(box > 0 && cutoff > 0, "box and cutoff must be positive");
  if (center_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(positions && species && row_offsets && mixing && A && workspace, "null pointer argument");
  Y3B_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, "workspace must be 16-byte aligned");
  const bool f64 = dtype == Y3B_F64;
  const size_t real = f64 ? sizeof(double) : sizeof(float);
  const int W2 = int(2 * (lmax + 1) * (lmax + 1));
  const int64_t per_atom = int64_t(W2) * Kp * int64_t(real);
  const int64_t chunk = workspace_bytes / per_atom;
  if (chunk < 1)
    return fail(Y3B_ERR_WORKSPACE, "ace_density_mixed_split: workspace below one atom (%lld bytes)",
                (long long)per_atom);
  const ShNorm nrm = make_sh_norm();
  cudaStream_t s = as_stream(stream);
  const int C = int(channel_count), S = int(species_count);
  // the product kernel's launch shape
  size_t prod_smem = 0;
  int per_sm = 1;
  if (f64) {
    prod_smem = size_t(S) * Kp * (C + 8) * sizeof(double);
    per_sm = int(std::max<size_t>(1, std::min<size_t>(4, size_t(220 * 1024) / (prod_smem + 1024))));
    Y3B_CUDA_TRY(cudaFuncSetAttribute(mixing_f64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(prod_smem)));
  } else {
    // residency: at most 512 / cols CTAs per SM, so that every CTA's tensor memory fits
    const size_t need = size_t(2 * kTcRows + 2 * Np) * Kp * sizeof(float);
    per_sm = 512 / cols < 4 ? 512 / cols : 4;
    const size_t floor_bytes = size_t(228 * 1024) / size_t(per_sm + 1) + 1024;
    prod_smem = need > floor_bytes ? need : floor_bytes;
    Y3B_CHECK_ARG(prod_smem <= 200 * 1024, "mixing operands need %zu bytes of shared memory", prod_smem);
    Y3B_CUDA_TRY(cudaFuncSetAttribute(mixing_tf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(prod_smem)));
  }
  for (int64_t a0 = 0; a0 < center_count; a0 += chunk) {
    const int64_t n = center_count - a0 < chunk ? center_count - a0 : chunk;
    const int grid_s = int(std::min<int64_t>((n + kSpWarps - 1) / kSpWarps, int64_t(kSMs) * 32));
    const size_t sp_smem = size_t(kSpWarps) * (W2 / 2) * (Kp + 1) * real;
#define Y3B_SP_CASE(T, L)                                                                                     \
  case L:                                                                                                     \
    Y3B_CUDA_TRY(cudaFuncSetAttribute(ace_species_density_kernel<T, L>,                                       \
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, int(sp_smem)));            \
    ace_species_density_kernel<T, L><<<grid_s, 32 * kSpWarps, sp_smem, s>>>(                                  \
        positions, species, atom_count, center_begin, a0, n, box, row_offsets, neighbors, S, int(nmax), Kp,  \
        T(cutoff), T(lambda), nrm, static_cast<T*>(workspace), status);                                       \
    break;
#define Y3B_SP_L(T)                                                                                           \
  switch (lmax) {                                                                                             \
    Y3B_SP_CASE(T, 0)                                                                                         \
    Y3B_SP_CASE(T, 1)                                                                                         \
    Y3B_SP_CASE(T, 2)                                                                                         \
    Y3B_SP_CASE(T, 3)                                                                                         \
    Y3B_SP_CASE(T, 4)                                                                                         \
    default:                                                                                                  \
      return fail(Y3B_ERR_UNSUPPORTED, "ace_density_mixed_split: lmax %lld not built (0..4)", (long long)lmax); \
  }
    if (f64) {
      Y3B_SP_L(double)
    } else {
      Y3B_SP_L(float)
    }
#undef Y3B_SP_L
#undef Y3B_SP_CASE
    Y3B_LAUNCH_CHECK();
    if (f64) {
      const int64_t tasks = n * ((W2 + 7) / 8);
      const int grid_t = int(std::min<int64_t>((tasks + kF64Warps - 1) / kF64Warps, int64_t(kSMs) * per_sm));
      mixing_f64_kernel<<<grid_t, 32 * kF64Warps, prod_smem, s>>>(
          static_cast<const double*>(workspace), n, W2, Kp, static_cast<const double*>(mixing), S, C, int(nmax),
          species + center_begin + a0, static_cast<double*>(A) + a0 * C * W2, status);
    } else {
      const int64_t tiles = (n * W2 + kTcRows - 1) / kTcRows;
      const int grid_t = int(std::min<int64_t>(tiles, int64_t(kSMs) * per_sm));
      mixing_tf32_kernel<<<grid_t, kTcThreads, prod_smem, s>>>(
          static_cast<const float*>(workspace), n, W2, Kp, static_cast<const float*>(mixing), S, C, int(nmax), Np,
          cols, species + center_begin + a0, static_cast<float*>(A) + a0 * C * W2, status);
    }
    Y3B_LAUNCH_CHECK();
  }
  return Y3B_OK;
}
