// Density accumulation without floating-point atomics.
//
// The reference CUDA kernel (execution_plan_cuda.cu:281-301) adds every edge
// row into its centre with global atomics, so its sums depend on scheduling.
// Here edges are bucketed into CSR rows with integer counting only, each row
// is put back into edge-index order, and one warp sums each output row in
// that order: results are bit-stable run to run.
#include "common.cuh"

namespace y3b {

constexpr int kScanThreads = 1024;

__global__ void count_centers_kernel(const int64_t* __restrict__ centers, int64_t E, int64_t N,
                                     unsigned long long* __restrict__ counts, int32_t* status) {
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < E;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t c = centers[e];
    if (c >= 0 && c < N) {
      atomicAdd(counts + c + 1, 1ull);
    } else if (status) {
      atomicOr(status, Y3B_STATUS_INDEX_RANGE);
    }
  }
}

// In-place inclusive scan of n int64 values with one CTA: each thread scans a
// contiguous chunk, chunk totals are scanned in shared memory, then added back.
__global__ void __launch_bounds__(kScanThreads) inclusive_scan_kernel(int64_t* __restrict__ a, int64_t n) {
  __shared__ int64_t sums[kScanThreads];
  const int t = threadIdx.x;
  const int64_t chunk = (n + kScanThreads - 1) / kScanThreads;
  const int64_t b = t * chunk, e = min(n, b + chunk);
  int64_t s = 0;
  for (int64_t i = b; i < e; ++i) s += a[i];
  sums[t] = s;
  __syncthreads();
  for (int off = 1; off < kScanThreads; off <<= 1) {
    const int64_t v = t >= off ? sums[t - off] : 0;
    __syncthreads();
    sums[t] += v;
    __syncthreads();
  }
  int64_t run = t > 0 ? sums[t - 1] : 0;
  for (int64_t i = b; i < e; ++i) {
    run += a[i];
    a[i] = run;
  }
}

__global__ void fill_rows_kernel(const int64_t* __restrict__ centers, int64_t E, int64_t N,
                                 const int64_t* __restrict__ row_off, int32_t* __restrict__ cursor,
                                 int64_t* __restrict__ order) {
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < E;
       e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t c = centers[e];
    if (c < 0 || c >= N) continue;
    const int slot = atomicAdd(cursor + c, 1);
    order[row_off[c] + slot] = e;
  }
}

// Restore edge-index order inside each row.  One warp per row: each lane
// ranks its elements against the whole row (rank = number of smaller edge
// indices; indices are distinct), then scatters them to their rank.
__global__ void sort_rows_kernel(const int64_t* __restrict__ row_off, int64_t N,
                                 int64_t* __restrict__ order, int64_t* __restrict__ scratch_order) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t i = warp; i < N; i += nwarps) {
    const int64_t b = row_off[i], e = row_off[i + 1];
    const int64_t len = e - b;
    if (len <= 1) continue;
    for (int64_t k = b + lane; k < e; k += 32) {
      const int64_t v = order[k];
      int64_t rank = 0;
      for (int64_t j = b; j < e; ++j) rank += order[j] < v;
      scratch_order[b + rank] = v;
    }
    __syncwarp();
    for (int64_t k = b + lane; k < e; k += 32) order[k] = scratch_order[k];
    __syncwarp();
  }
}

// One warp per output row; lanes over channels; edges of the row in order.
template <typename T>
__global__ void __launch_bounds__(256) csr_accumulate_kernel(const T* __restrict__ v,
                                                             const int64_t* __restrict__ row_off,
                                                             const int64_t* __restrict__ order,
                                                             int64_t N, int64_t C, T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t i = warp; i < N; i += nwarps) {
    const int64_t b = row_off[i], e = row_off[i + 1];
    for (int64_t c0 = 0; c0 < C; c0 += 32) {
      const int64_t c = c0 + lane;
      if (c >= C) break;
      T acc = zero<T>();
      for (int64_t k = b; k < e; ++k) {
        const int64_t src = order ? order[k] : k;
        acc = add(acc, v[src * C + c]);
      }
      out[i * C + c] = acc;
    }
  }
}

template <typename T>
__global__ void adjoint_kernel(const T* __restrict__ adj, const int64_t* __restrict__ centers, int64_t E,
                               int64_t C, int64_t N, T* __restrict__ out, int32_t* status) {
  const int64_t total = E * C;
  for (int64_t lin = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; lin < total;
       lin += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = lin / C, c = lin - e * C;
    const int64_t i = centers[e];
    if (i >= 0 && i < N) {
      out[lin] = adj[i * C + c];
    } else {
      out[lin] = zero<T>();
      if (status) atomicOr(status, Y3B_STATUS_INDEX_RANGE);
    }
  }
}

inline int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

struct DensityWorkspace {
  int64_t* row_off;   // [N+1]
  int32_t* cursor;    // [N]
  int64_t* order;     // [E]
  int64_t* scratch;   // [E]
  int64_t bytes;
};

inline DensityWorkspace carve(void* base, int64_t E, int64_t N) {
  DensityWorkspace w;
  char* p = static_cast<char*>(base);
  int64_t off = 0;
  w.row_off = reinterpret_cast<int64_t*>(p + off); off += align256((N + 1) * 8);
  w.cursor = reinterpret_cast<int32_t*>(p + off); off += align256(N * 4);
  w.order = reinterpret_cast<int64_t*>(p + off); off += align256(E * 8);
  w.scratch = reinterpret_cast<int64_t*>(p + off); off += align256(E * 8);
  w.bytes = off;
  return w;
}

}  // namespace y3b

using namespace y3b;

extern "C" int64_t y3b_density_accumulate_workspace_bytes(int64_t edge_count, int64_t atom_count) {
  if (edge_count < 0 || atom_count < 0) return -1;
  return carve(nullptr, edge_count, atom_count).bytes;
}

namespace y3b {
// Shared by the allocating entry point and callers that own the workspace.
int density_accumulate_impl(int dtype, const void* edge_values, const int64_t* centers, int64_t E,
                            int64_t C, int64_t N, void* workspace, int64_t workspace_bytes, void* out,
                            int32_t* status, cudaStream_t s) {
  Y3B_CHECK_ARG(E >= 0 && C >= 0 && N >= 0, "negative size");
  Y3B_CHECK_ARG(E < (int64_t(1) << 31) * 16, "edge count too large");
  if (N == 0 || C == 0) return Y3B_OK;
  Y3B_CHECK_ARG(out != nullptr, "null output");
  const DensityWorkspace w = carve(workspace, E, N);
  Y3B_CHECK_ARG(workspace != nullptr && workspace_bytes >= w.bytes,
                "workspace too small: need %lld bytes, got %lld", (long long)w.bytes,
                (long long)workspace_bytes);
  Y3B_CHECK_ARG(E == 0 || (edge_values && centers), "null input");
  Y3B_CUDA_TRY(cudaMemsetAsync(w.row_off, 0, (N + 1) * 8, s));
  Y3B_CUDA_TRY(cudaMemsetAsync(w.cursor, 0, N * 4, s));
  if (E > 0) {
    count_centers_kernel<<<grid_for(E, 256), 256, 0, s>>>(
        centers, E, N, reinterpret_cast<unsigned long long*>(w.row_off), status);
    Y3B_LAUNCH_CHECK();
  }
  inclusive_scan_kernel<<<1, kScanThreads, 0, s>>>(w.row_off, N + 1);
  Y3B_LAUNCH_CHECK();
  if (E > 0) {
    fill_rows_kernel<<<grid_for(E, 256), 256, 0, s>>>(centers, E, N, w.row_off, w.cursor, w.order);
    Y3B_LAUNCH_CHECK();
    sort_rows_kernel<<<grid_for(N * 32, 256), 256, 0, s>>>(w.row_off, N, w.order, w.scratch);
    Y3B_LAUNCH_CHECK();
  }
  Y3B_DISPATCH(dtype, T, {
    csr_accumulate_kernel<T><<<grid_for(N * 32, 256), 256, 0, s>>>(
        static_cast<const T*>(edge_values), w.row_off, w.order, N, C, static_cast<T*>(out));
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}
}  // namespace y3b

extern "C" int y3b_density_accumulate(int dtype, const void* edge_values, const int64_t* centers,
                                      int64_t edge_count, int64_t channel_count, int64_t atom_count,
                                      void* workspace, int64_t workspace_bytes, void* out,
                                      int32_t* status, void* stream) {
  return density_accumulate_impl(dtype, edge_values, centers, edge_count, channel_count, atom_count,
                                 workspace, workspace_bytes, out, status, as_stream(stream));
}

extern "C" int y3b_density_accumulate_csr(int dtype, const void* edge_values,
                                          const int64_t* row_offsets, const int64_t* edge_order,
                                          int64_t atom_count, int64_t channel_count, void* out,
                                          void* stream) {
  Y3B_CHECK_ARG(atom_count >= 0 && channel_count >= 0, "negative size");
  if (atom_count == 0 || channel_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(row_offsets && out, "null pointer argument");
  Y3B_DISPATCH(dtype, T, {
    csr_accumulate_kernel<T><<<grid_for(atom_count * 32, 256), 256, 0, as_stream(stream)>>>(
        static_cast<const T*>(edge_values), row_offsets, edge_order, atom_count, channel_count,
        static_cast<T*>(out));
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}

extern "C" int y3b_density_accumulate_adjoint(int dtype, const void* atomic_adjoint,
                                              const int64_t* centers, int64_t edge_count,
                                              int64_t channel_count, int64_t atom_count,
                                              void* edge_adjoint, int32_t* status, void* stream) {
  Y3B_CHECK_ARG(edge_count >= 0 && channel_count >= 0 && atom_count >= 0, "negative size");
  if (edge_count == 0 || channel_count == 0) return Y3B_OK;
  Y3B_CHECK_ARG(atomic_adjoint && centers && edge_adjoint, "null pointer argument");
  Y3B_DISPATCH(dtype, T, {
    adjoint_kernel<T><<<grid_for(edge_count * channel_count, 256), 256, 0, as_stream(stream)>>>(
        static_cast<const T*>(atomic_adjoint), centers, edge_count, channel_count, atom_count,
        static_cast<T*>(edge_adjoint), status);
  });
  Y3B_LAUNCH_CHECK();
  return Y3B_OK;
}
