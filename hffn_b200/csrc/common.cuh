// Shared device helpers of the HFFN sm_100a kernels: exact GELU and its derivative, warp reductions, float/bf16
// storage conversions, and the host-side status plumbing of the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "../../include/hffn_b200.h"

namespace hffn {

// Exact GELU, 0.5 z (1 + erf(z / sqrt 2)): the reference's `gelu` (kernels.py:87-89), CUDA's erff.
__device__ __forceinline__ float gelu(float z) { return 0.5f * z * (1.0f + erff(z * 0.70710678118654752f)); }

// d gelu / dz = 0.5 (1 + erf(z / sqrt 2)) + z exp(-z^2 / 2) / sqrt(2 pi): the reference's `gelu_grad`
// (kernels_train.py:102-104), PyTorch's GELU backward with approximate="none"; CUDA's erff and expf.
__device__ __forceinline__ float gelu_grad(float z) {
  return 0.5f * (1.0f + erff(z * 0.70710678118654752f)) + z * 0.39894228040143268f * expf(-0.5f * z * z);
}

// xor-shuffle tree 16, 8, 4, 2, 1: every lane ends with the same sum, in the same order on every lane.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
  return v;
}

// Storage types: float (fp32 path) or __nv_bfloat16 (bf16 path); arithmetic is always fp32.
template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

template <typename T> __device__ __forceinline__ T ldg(const T* p) { return __ldg(p); }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Internal status (never returned by the C ABI): a specialised launcher declines a call, the general one runs it.
constexpr int kNotApplicable = -1000;

// Per-thread last error message of the C ABI (hffn_last_error).
void set_error(const char* fmt, ...);
const char* last_error();

// Status of the last launch on the calling thread.
inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return HFFN_ERR_CUDA;
  }
  return HFFN_OK;
}

// Make the device of `stream` current for the launches of one call (a null stream keeps the current device). A stream
// being captured into a CUDA graph is left as it is: the capture runs on the current device, and device queries and
// switches are not permitted during a capture.
inline int bind_stream_device(void* stream) {
  if (stream == nullptr) return HFFN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &capture) == cudaSuccess && capture != cudaStreamCaptureStatusNone) return HFFN_OK;
  int device = -1, current = -1;
  cudaError_t e = cudaStreamGetDevice(s, &device);
  if (e == cudaSuccess) e = cudaGetDevice(&current);
  if (e == cudaSuccess && device != current) e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    set_error("stream device: %s", cudaGetErrorString(e));
    return HFFN_ERR_CUDA;
  }
  return HFFN_OK;
}

}  // namespace hffn

#define HFFN_REQUIRE(cond, ...)            \
  do {                                     \
    if (!(cond)) {                         \
      ::hffn::set_error(__VA_ARGS__);      \
      return HFFN_ERR_ARGUMENT;            \
    }                                      \
  } while (0)

#define HFFN_TRY(expr)               \
  do {                               \
    int _status = (expr);            \
    if (_status != HFFN_OK) return _status; \
  } while (0)
