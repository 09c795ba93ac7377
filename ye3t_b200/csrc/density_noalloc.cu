// Density accumulation for callers that cannot allocate device memory.
//
// Some hosts of this library own every byte of device memory themselves and
// forbid allocation once they are running: a molecular-dynamics engine that
// calls the density from its per-timestep force loop, for example, or a
// serving process that reserves all memory at start-up.  cudaMalloc there
// would synchronise the device, can fail in the middle of a run, and may not
// be permitted at all.  y3b_density_accumulate_noalloc gives those callers
// the same deterministic result as y3b_density_accumulate without asking
// them for a workspace: its scratch is the fixed array below, which every
// GPU that loads the library holds until the process exits.
//
// The array is shared by all calls on a device and keeps whatever the last
// call left in it.  The counting arrays are cleared at the start of each
// call; the ordering arrays are fully rewritten.  Calls whose execution
// overlaps on the GPU (different streams, or several host threads) race on
// the array and must be serialised by the caller.
#include <mutex>

#include "common.cuh"

namespace y3b {

int density_accumulate_impl(int dtype, const void* edge_values, const int64_t* centers, int64_t E,
                            int64_t C, int64_t N, void* workspace, int64_t workspace_bytes, void* out,
                            int32_t* status, cudaStream_t s);

namespace {

constexpr int64_t kScratchBytes = Y3B_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_density_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of g_density_scratch on the current device.  In host code
// the symbol name is only a host-side handle, so the address is looked up
// once per device with that device current and cached.
int scratch_address(void** out) {
  int dev = -1;
  Y3B_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(Y3B_ERR_UNSUPPORTED, "density_accumulate_noalloc: device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_density_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(Y3B_ERR_CUDA, "density_accumulate_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    g_scratch_address[dev] = p;
  }
  *out = g_scratch_address[dev];
  return Y3B_OK;
}

}  // namespace
}  // namespace y3b

using namespace y3b;

extern "C" int y3b_density_accumulate_noalloc(int dtype, const void* edge_values, const int64_t* centers,
                                              int64_t edge_count, int64_t channel_count,
                                              int64_t atom_count, void* out, int32_t* status,
                                              void* stream) {
  const int64_t need = y3b_density_accumulate_workspace_bytes(edge_count, atom_count);
  Y3B_CHECK_ARG(need >= 0, "density_accumulate_noalloc: negative size");
  if (need > kScratchBytes)
    return fail(Y3B_ERR_WORKSPACE,
                "density_accumulate_noalloc: %lld edges and %lld atoms need %lld bytes of scratch, more "
                "than its fixed %lld-byte array; use y3b_density_accumulate with a caller workspace",
                (long long)edge_count, (long long)atom_count, (long long)need, (long long)kScratchBytes);
  void* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  return density_accumulate_impl(dtype, edge_values, centers, edge_count, channel_count, atom_count,
                                 scratch, kScratchBytes, out, status, as_stream(stream));
}
