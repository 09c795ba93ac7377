// Cubic periodic cell-list neighbour builder producing sorted CSR rows.
//
// The reference has no neighbour-list code (applications supply the density
// factors); this is the builder the fused A-basis path consumes.  The
// minimum-image displacement and the r^2 <= rc^2 test use non-contracting
// intrinsics so every pair decision and displacement is bit-identical to the
// serial CPU oracle.
#include "common.cuh"
#include "neighbors.cuh"

namespace y3b {

namespace {

struct CellWorkspace {
  int64_t* cell_start;  // [nc + 1]
  int32_t* cursor;      // [nc]
  int32_t* atom_cell;   // [N]
  int32_t* cell_atoms;  // [N]
  int64_t* block_sums;  // [kScanBlocks]: segment totals of the prefix sums
  int64_t bytes;
};

constexpr int kScanBlocks = 256;   // segments of a prefix sum, one CTA each
constexpr int kScanThreads = 256;

inline int64_t al(int64_t x) { return (x + 255) & ~int64_t(255); }

inline CellWorkspace carve_cells(void* base, int64_t N, int64_t nc) {
  CellWorkspace w;
  char* p = static_cast<char*>(base);
  int64_t o = 0;
  w.cell_start = reinterpret_cast<int64_t*>(p + o); o += al((nc + 1) * 8);
  w.cursor = reinterpret_cast<int32_t*>(p + o); o += al(nc * 4);
  w.atom_cell = reinterpret_cast<int32_t*>(p + o); o += al(N * 4);
  w.cell_atoms = reinterpret_cast<int32_t*>(p + o); o += al(N * 4);
  w.block_sums = reinterpret_cast<int64_t*>(p + o); o += al(kScanBlocks * 8);
  w.bytes = o;
  return w;
}

__device__ __forceinline__ int cell_coord(double x, double box, int n) {
  double f = x / box;
  f -= floor(f);
  int c = int(f * n);
  return c < 0 ? 0 : (c >= n ? n - 1 : c);
}

// A window of z cell layers [zb, zb + zc) (periodic; zc == n is the whole
// box): only atoms inside it are binned, in window-local cells
// ((z - zb) mod n, y, x).  Returns -1 for a z layer outside the window.
__device__ __forceinline__ int window_z(int cz, int n, int zb, int zc) {
  const int wz = (cz - zb + n) % n;
  return wz < zc ? wz : -1;
}

__global__ void assign_cells_kernel(const double* __restrict__ pos, int64_t N, double box, int n, int zb, int zc,
                                    int32_t* __restrict__ atom_cell,
                                    unsigned long long* __restrict__ counts) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < N;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int cx = cell_coord(pos[3 * i], box, n), cy = cell_coord(pos[3 * i + 1], box, n),
              wz = window_z(cell_coord(pos[3 * i + 2], box, n), n, zb, zc);
    if (wz < 0) {
      atom_cell[i] = -1;
      continue;
    }
    const int c = (wz * n + cy) * n + cx;
    atom_cell[i] = c;
    atomicAdd(counts + c + 1, 1ull);
  }
}

__global__ void fill_cells_kernel(int64_t N, const int32_t* __restrict__ atom_cell,
                                  const int64_t* __restrict__ cell_start, int32_t* __restrict__ cursor,
                                  int32_t* __restrict__ cell_atoms) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < N;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int c = atom_cell[i];
    if (c < 0) continue;
    const int slot = atomicAdd(cursor + c, 1);
    cell_atoms[cell_start[c] + slot] = int32_t(i);
  }
}

// Insertion sort of each cell's members (cells hold a handful of atoms).
__global__ void sort_cells_kernel(int64_t nc, const int64_t* __restrict__ cell_start,
                                  int32_t* __restrict__ cell_atoms) {
  for (int64_t c = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; c < nc;
       c += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = cell_start[c], e = cell_start[c + 1];
    for (int64_t k = b + 1; k < e; ++k) {
      const int32_t v = cell_atoms[k];
      int64_t j = k - 1;
      while (j >= b && cell_atoms[j] > v) {
        cell_atoms[j + 1] = cell_atoms[j];
        --j;
      }
      cell_atoms[j + 1] = v;
    }
  }
}

// Visit every candidate neighbour j of centre i exactly once.  A centre whose
// neighbouring z layers leave the binned window returns false (its row is
// incomplete); the caller reports it.
template <typename F>
__device__ __forceinline__ bool for_each_neighbor(const double* __restrict__ pos, int64_t i, double box,
                                                  double rc2, int n, int zb, int zc,
                                                  const int64_t* __restrict__ cell_start,
                                                  const int32_t* __restrict__ cell_atoms, F&& f) {
  const double xi = pos[3 * i], yi = pos[3 * i + 1], zi = pos[3 * i + 2];
  const int span = n >= 3 ? 1 : 0;
  const int cx = cell_coord(xi, box, n), cy = cell_coord(yi, box, n), cz = cell_coord(zi, box, n);
  bool inside = true;
  for (int dz = -span; dz <= span; ++dz) {
    const int wz = window_z((cz + dz + n) % n, n, zb, zc);
    if (wz < 0) {
      inside = false;
      continue;
    }
    for (int dy = -span; dy <= span; ++dy)
      for (int dx = -span; dx <= span; ++dx) {
        const int x = (cx + dx + n) % n, y = (cy + dy + n) % n;
        const int c = (wz * n + y) * n + x;
        for (int64_t k = cell_start[c]; k < cell_start[c + 1]; ++k) {
          const int32_t j = cell_atoms[k];
          if (j == i) continue;
          double d[3];
          min_image(pos, i, j, box, d);
          if (dist2(d) <= rc2) f(j);
        }
      }
  }
  return inside;
}

__global__ void count_neighbors_kernel(const double* __restrict__ pos, int64_t begin, int64_t end,
                                       double box, double rc2, int n, int zb, int zc,
                                       const int64_t* __restrict__ cell_start,
                                       const int32_t* __restrict__ cell_atoms,
                                       int64_t* __restrict__ row_offsets, int32_t* status) {
  for (int64_t i = begin + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < end;
       i += int64_t(gridDim.x) * blockDim.x) {
    int64_t cnt = 0;
    if (!for_each_neighbor(pos, i, box, rc2, n, zb, zc, cell_start, cell_atoms, [&](int32_t) { ++cnt; }) &&
        status)
      atomicOr(status, Y3B_STATUS_INDEX_RANGE);
    row_offsets[i - begin + 1] = cnt;
    if (i == begin) row_offsets[0] = 0;
  }
}

__global__ void fill_neighbors_kernel(const double* __restrict__ pos, int64_t begin, int64_t end,
                                      double box, double rc2, int n, int zb, int zc,
                                      const int64_t* __restrict__ cell_start,
                                      const int32_t* __restrict__ cell_atoms,
                                      const int64_t* __restrict__ row_offsets, int64_t capacity,
                                      int32_t* __restrict__ nbr, int32_t* status) {
  for (int64_t i = begin + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < end;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = row_offsets[i - begin];
    int64_t e = row_offsets[i - begin + 1];
    if (e > capacity) {
      if (status) atomicOr(status, Y3B_STATUS_CAPACITY);
      e = capacity;
    }
    int64_t k = b;
    for_each_neighbor(pos, i, box, rc2, n, zb, zc, cell_start, cell_atoms, [&](int32_t j) {
      if (k < e) nbr[k] = j;
      ++k;
    });
    for (int64_t a = b + 1; a < e; ++a) {  // rows in increasing neighbour index
      const int32_t v = nbr[a];
      int64_t q = a - 1;
      while (q >= b && nbr[q] > v) {
        nbr[q + 1] = nbr[q];
        --q;
      }
      nbr[q + 1] = v;
    }
  }
}

// In-place inclusive prefix sum of n int64 values in two launches over kScanBlocks
// segments of ceil(n / kScanBlocks) values: the segments' totals, then each segment
// scanned in tiles of kScanThreads values (warp shuffles, then the warps' totals),
// starting from the total of the segments before it.  Coalesced and exact.
__device__ __forceinline__ int64_t block_inclusive_scan(int64_t v, int64_t* warp_tot, int64_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  int64_t before = 0;
  total = 0;
  for (int w = 0; w < kScanThreads / 32; ++w) {
    if (w < warp) before += warp_tot[w];
    total += warp_tot[w];
  }
  __syncthreads();
  return before + v;
}

__global__ void __launch_bounds__(kScanThreads) scan_sums_kernel(const int64_t* __restrict__ a, int64_t n,
                                                                 int64_t seg, int64_t* __restrict__ sums) {
  __shared__ int64_t warp_tot[kScanThreads / 32];
  const int64_t b = blockIdx.x * seg, e = b + seg < n ? b + seg : n;
  int64_t s = 0;
  for (int64_t i = b + threadIdx.x; i < e; i += kScanThreads) s += a[i];
  int64_t total;
  block_inclusive_scan(s, warp_tot, total);
  if (threadIdx.x == 0) sums[blockIdx.x] = total;
}

__global__ void __launch_bounds__(kScanThreads) scan_apply_kernel(int64_t* __restrict__ a, int64_t n, int64_t seg,
                                                                  const int64_t* __restrict__ sums) {
  __shared__ int64_t warp_tot[kScanThreads / 32];
  int64_t carry;  // the total of the segments before this one
  block_inclusive_scan(threadIdx.x < blockIdx.x ? sums[threadIdx.x] : 0, warp_tot, carry);
  const int64_t b = blockIdx.x * seg, e = b + seg < n ? b + seg : n;
  for (int64_t t = b; t < e; t += kScanThreads) {
    const int64_t i = t + threadIdx.x;
    int64_t tile;
    const int64_t v = block_inclusive_scan(i < e ? a[i] : 0, warp_tot, tile);
    if (i < e) a[i] = carry + v;
    carry += tile;
  }
}

void scan_i64(int64_t* a, int64_t n, int64_t* sums, cudaStream_t s) {
  const int64_t seg = (n + kScanBlocks - 1) / kScanBlocks;
  scan_sums_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(a, n, seg, sums);
  scan_apply_kernel<<<kScanBlocks, kScanThreads, 0, s>>>(a, n, seg, sums);
}

}  // namespace

int cells_per_side(double box, double cutoff) {
  if (!(box > 0) || !(cutoff > 0)) return 1;
  const double r = box / cutoff;
  if (r < 3.0) return 1;
  return int(r > 1024.0 ? 1024.0 : r);
}

}  // namespace y3b

using namespace y3b;

extern "C" int64_t y3b_neighbor_workspace_bytes(int64_t atom_count, double box, double cutoff) {
  const int64_t n = cells_per_side(box, cutoff);
  return carve_cells(nullptr, atom_count, n * n * n).bytes;
}

namespace {

// z window of the cell list: zc >= n (or a box of fewer than 3 cells) bins the
// whole box.
void clamp_window(int n, int64_t z_begin, int64_t z_count, int& zb, int& zc) {
  if (z_count <= 0 || z_count >= n || n < 3) {
    zb = 0;
    zc = n;
  } else {
    zb = int(((z_begin % n) + n) % n);
    zc = int(z_count);
  }
}

int neighbor_count_impl(const double* positions, int64_t atom_count, int64_t center_begin, int64_t center_end,
                        double box, double cutoff, int64_t z_begin, int64_t z_count, void* workspace,
                        int64_t workspace_bytes, int64_t* row_offsets, int32_t* status, cudaStream_t s) {
  Y3B_CHECK_ARG(atom_count >= 0 && atom_count < (int64_t(1) << 31), "atom count out of range");
  Y3B_CHECK_ARG(0 <= center_begin && center_begin <= center_end && center_end <= atom_count,
                "bad centre range [%lld, %lld)", (long long)center_begin, (long long)center_end);
  Y3B_CHECK_ARG(box > 0 && cutoff > 0, "box and cutoff must be positive");
  Y3B_CHECK_ARG(row_offsets != nullptr, "null row_offsets");
  if (center_end == center_begin) {
    Y3B_CUDA_TRY(cudaMemsetAsync(row_offsets, 0, 8, s));
    return Y3B_OK;
  }
  Y3B_CHECK_ARG(positions != nullptr, "null positions");
  const int n = cells_per_side(box, cutoff);
  int zb = 0, zc = n;
  clamp_window(n, z_begin, z_count, zb, zc);
  const int64_t nc = int64_t(zc) * n * n;
  const CellWorkspace w = carve_cells(workspace, atom_count, nc);
  Y3B_CHECK_ARG(workspace && workspace_bytes >= w.bytes, "neighbour workspace too small: need %lld",
                (long long)w.bytes);
  Y3B_CUDA_TRY(cudaMemsetAsync(w.cell_start, 0, (nc + 1) * 8, s));
  Y3B_CUDA_TRY(cudaMemsetAsync(w.cursor, 0, nc * 4, s));
  assign_cells_kernel<<<grid_for(atom_count, 256), 256, 0, s>>>(
      positions, atom_count, box, n, zb, zc, w.atom_cell, reinterpret_cast<unsigned long long*>(w.cell_start));
  Y3B_LAUNCH_CHECK();
  scan_i64(w.cell_start, nc + 1, w.block_sums, s);
  Y3B_LAUNCH_CHECK();
  fill_cells_kernel<<<grid_for(atom_count, 256), 256, 0, s>>>(atom_count, w.atom_cell, w.cell_start,
                                                              w.cursor, w.cell_atoms);
  Y3B_LAUNCH_CHECK();
  sort_cells_kernel<<<grid_for(nc, 256), 256, 0, s>>>(nc, w.cell_start, w.cell_atoms);
  Y3B_LAUNCH_CHECK();
  const int64_t count = center_end - center_begin;
  count_neighbors_kernel<<<grid_for(count, 128), 128, 0, s>>>(
      positions, center_begin, center_end, box, cutoff * cutoff, n, zb, zc, w.cell_start, w.cell_atoms,
      row_offsets, status);
  Y3B_LAUNCH_CHECK();
  scan_i64(row_offsets, count + 1, w.block_sums, s);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

int neighbor_fill_impl(const double* positions, int64_t atom_count, int64_t center_begin, int64_t center_end,
                       double box, double cutoff, int64_t z_begin, int64_t z_count, const void* workspace,
                       int64_t workspace_bytes, const int64_t* row_offsets, int64_t capacity, int32_t* neighbors,
                       int32_t* status, cudaStream_t s) {
  Y3B_CHECK_ARG(0 <= center_begin && center_begin <= center_end && center_end <= atom_count,
                "bad centre range");
  if (center_end == center_begin) return Y3B_OK;
  Y3B_CHECK_ARG(positions && row_offsets && neighbors, "null pointer argument");
  Y3B_CHECK_ARG(capacity >= 0, "negative neighbour capacity");
  const int n = cells_per_side(box, cutoff);
  int zb = 0, zc = n;
  clamp_window(n, z_begin, z_count, zb, zc);
  const int64_t nc = int64_t(zc) * n * n;
  const CellWorkspace w = carve_cells(const_cast<void*>(workspace), atom_count, nc);
  Y3B_CHECK_ARG(workspace && workspace_bytes >= w.bytes, "neighbour workspace too small");
  const int64_t count = center_end - center_begin;
  fill_neighbors_kernel<<<grid_for(count, 128), 128, 0, s>>>(
      positions, center_begin, center_end, box, cutoff * cutoff, n, zb, zc, w.cell_start, w.cell_atoms,
      row_offsets, capacity, neighbors, status);
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

}  // namespace

extern "C" int y3b_neighbor_count(const double* positions, int64_t atom_count, int64_t center_begin,
                                  int64_t center_end, double box, double cutoff, void* workspace,
                                  int64_t workspace_bytes, int64_t* row_offsets, void* stream) {
  return neighbor_count_impl(positions, atom_count, center_begin, center_end, box, cutoff, 0, 0, workspace,
                             workspace_bytes, row_offsets, nullptr, as_stream(stream));
}

extern "C" int y3b_neighbor_fill(const double* positions, int64_t atom_count, int64_t center_begin,
                                 int64_t center_end, double box, double cutoff, const void* workspace,
                                 int64_t workspace_bytes, const int64_t* row_offsets, int32_t* neighbors,
                                 void* stream) {
  return neighbor_fill_impl(positions, atom_count, center_begin, center_end, box, cutoff, 0, 0, workspace,
                            workspace_bytes, row_offsets, INT64_MAX, neighbors, nullptr, as_stream(stream));
}

extern "C" int y3b_neighbor_count_window(const double* positions, int64_t atom_count, int64_t center_begin,
                                         int64_t center_end, double box, double cutoff, int64_t z_cell_begin,
                                         int64_t z_cell_count, void* workspace, int64_t workspace_bytes,
                                         int64_t* row_offsets, int32_t* status, void* stream) {
  return neighbor_count_impl(positions, atom_count, center_begin, center_end, box, cutoff, z_cell_begin,
                             z_cell_count, workspace, workspace_bytes, row_offsets, status, as_stream(stream));
}

extern "C" int y3b_neighbor_fill_window(const double* positions, int64_t atom_count, int64_t center_begin,
                                        int64_t center_end, double box, double cutoff, int64_t z_cell_begin,
                                        int64_t z_cell_count, const void* workspace, int64_t workspace_bytes,
                                        const int64_t* row_offsets, int64_t neighbor_capacity,
                                        int32_t* neighbors, int32_t* status, void* stream) {
  return neighbor_fill_impl(positions, atom_count, center_begin, center_end, box, cutoff, z_cell_begin,
                            z_cell_count, workspace, workspace_bytes, row_offsets, neighbor_capacity, neighbors,
                            status, as_stream(stream));
}

extern "C" int64_t y3b_neighbor_cells_per_side(double box, double cutoff) { return cells_per_side(box, cutoff); }
