// Error plumbing, ABI version and the FMA-throughput measurement kernel.
#include <cstdarg>
#include <cstring>

#include "common.cuh"

namespace y3b {

static thread_local std::string g_last_error;

void set_error(int code, const std::string& msg) {
  (void)code;
  g_last_error = msg;
}

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_error(code, buf);
  return code;
}

// Eight independent FMA chains per thread; the sink write keeps the chains
// live.  The operands stay in registers, so the kernel measures the FMA
// pipe, not memory.
template <typename T>
__global__ void fma_peak_kernel(T* sink, int iterations, T a, T b) {
  T x0 = T(threadIdx.x) * T(1e-7), x1 = x0 + T(1), x2 = x0 + T(2), x3 = x0 + T(3);
  T x4 = x0 + T(4), x5 = x0 + T(5), x6 = x0 + T(6), x7 = x0 + T(7);
#pragma unroll 4
  for (int i = 0; i < iterations; ++i) {
    x0 = fma(x0, a, b); x1 = fma(x1, a, b); x2 = fma(x2, a, b); x3 = fma(x3, a, b);
    x4 = fma(x4, a, b); x5 = fma(x5, a, b); x6 = fma(x6, a, b); x7 = fma(x7, a, b);
  }
  const T s = ((x0 + x1) + (x2 + x3)) + ((x4 + x5) + (x6 + x7));
  if (s == T(-12345.678)) sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

}  // namespace y3b

using namespace y3b;

extern "C" int32_t y3b_abi_version(void) { return Y3B_ABI_VERSION; }

extern "C" const char* y3b_last_error(void) { return g_last_error.c_str(); }

extern "C" int y3b_fma_peak_launch(int dtype, int32_t blocks, int32_t threads, int32_t iterations,
                                   void* sink, double* flops, void* stream) {
  Y3B_CHECK_ARG(blocks > 0 && threads > 0 && threads <= 1024 && iterations > 0,
                "bad launch shape %d x %d x %d", blocks, threads, iterations);
  Y3B_CHECK_ARG(sink != nullptr, "sink must hold blocks*threads values");
  if (dtype == Y3B_F64) {
    fma_peak_kernel<double><<<blocks, threads, 0, as_stream(stream)>>>(
        static_cast<double*>(sink), iterations, 0.999999, 1e-9);
  } else if (dtype == Y3B_F32) {
    fma_peak_kernel<float><<<blocks, threads, 0, as_stream(stream)>>>(
        static_cast<float*>(sink), iterations, 0.999999f, 1e-9f);
  } else {
    return fail(Y3B_ERR_ARGUMENT, "fma peak: dtype must be F32 or F64");
  }
  Y3B_LAUNCH_CHECK();
  if (flops) *flops = 2.0 * 8.0 * double(blocks) * double(threads) * double(iterations);
  return Y3B_OK;
}
