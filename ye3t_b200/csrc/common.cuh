// Shared device/host helpers for the ye3t_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>
#include <string>

#include "ye3t_b200.h"

namespace y3b {

constexpr int kSMs = 148;  // B200: 2 dies x 74 SMs

// ---------------------------------------------------------------------------
// Error reporting: every entry point returns a status code and records a
// message retrievable with y3b_last_error() (thread-local).
// ---------------------------------------------------------------------------
void set_error(int code, const std::string& msg);
int fail(int code, const char* fmt, ...);

#define Y3B_CHECK_ARG(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) return ::y3b::fail(Y3B_ERR_ARGUMENT, __VA_ARGS__); \
  } while (0)

#define Y3B_CUDA_TRY(expr)                                                             \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    if (_e != cudaSuccess)                                                             \
      return ::y3b::fail(Y3B_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                         __FILE__, __LINE__);                                          \
  } while (0)

#define Y3B_LAUNCH_CHECK() Y3B_CUDA_TRY(cudaGetLastError())

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int grid_for(int64_t work, int threads, int per_sm_blocks = 16) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = int64_t(kSMs) * per_sm_blocks * 8;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return int(g);
}

// ---------------------------------------------------------------------------
// Scalar traits: real (float, double) and complex (float2, double2).
// ---------------------------------------------------------------------------
template <typename T> struct Real { using type = T; };
template <> struct Real<float2> { using type = float; };
template <> struct Real<double2> { using type = double; };

template <typename T> __host__ __device__ __forceinline__ T zero();
template <> __host__ __device__ __forceinline__ float zero<float>() { return 0.f; }
template <> __host__ __device__ __forceinline__ double zero<double>() { return 0.0; }
template <> __host__ __device__ __forceinline__ float2 zero<float2>() { return make_float2(0.f, 0.f); }
template <> __host__ __device__ __forceinline__ double2 zero<double2>() { return make_double2(0.0, 0.0); }

template <typename T> __host__ __device__ __forceinline__ T one();
template <> __host__ __device__ __forceinline__ float one<float>() { return 1.f; }
template <> __host__ __device__ __forceinline__ double one<double>() { return 1.0; }
template <> __host__ __device__ __forceinline__ float2 one<float2>() { return make_float2(1.f, 0.f); }
template <> __host__ __device__ __forceinline__ double2 one<double2>() { return make_double2(1.0, 0.0); }

__host__ __device__ __forceinline__ float mul(float a, float b) { return a * b; }
__host__ __device__ __forceinline__ double mul(double a, double b) { return a * b; }
__host__ __device__ __forceinline__ float2 mul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__host__ __device__ __forceinline__ double2 mul(double2 a, double2 b) {
  return make_double2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__host__ __device__ __forceinline__ float add(float a, float b) { return a + b; }
__host__ __device__ __forceinline__ double add(double a, double b) { return a + b; }
__host__ __device__ __forceinline__ float2 add(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__host__ __device__ __forceinline__ double2 add(double2 a, double2 b) { return make_double2(a.x + b.x, a.y + b.y); }

// real x complex / real x real scaling
__host__ __device__ __forceinline__ double2 scale(double s, double2 a) { return make_double2(s * a.x, s * a.y); }
__host__ __device__ __forceinline__ float2 scale(float s, float2 a) { return make_float2(s * a.x, s * a.y); }
__host__ __device__ __forceinline__ double scale(double s, double a) { return s * a; }
__host__ __device__ __forceinline__ float scale(float s, float a) { return s * a; }

__host__ __device__ __forceinline__ double re(double a) { return a; }
__host__ __device__ __forceinline__ float re(float a) { return a; }
__host__ __device__ __forceinline__ double re(double2 a) { return a.x; }
__host__ __device__ __forceinline__ float re(float2 a) { return a.x; }

// Dispatch on the public dtype code (Y3B_F32 .. Y3B_C128).
#define Y3B_DISPATCH(dtype, T, ...)                                     \
  switch (dtype) {                                                      \
    case Y3B_F32: { using T = float; __VA_ARGS__; break; }              \
    case Y3B_F64: { using T = double; __VA_ARGS__; break; }             \
    case Y3B_C64: { using T = float2; __VA_ARGS__; break; }             \
    case Y3B_C128: { using T = double2; __VA_ARGS__; break; }           \
    default: return ::y3b::fail(Y3B_ERR_ARGUMENT, "unsupported dtype code %d", int(dtype)); \
  }

#define Y3B_DISPATCH_REAL(dtype, T, ...)                                \
  switch (dtype) {                                                      \
    case Y3B_F32: { using T = float; __VA_ARGS__; break; }              \
    case Y3B_F64: { using T = double; __VA_ARGS__; break; }             \
    default: return ::y3b::fail(Y3B_ERR_ARGUMENT, "dtype code %d is not a real type", int(dtype)); \
  }

}  // namespace y3b
