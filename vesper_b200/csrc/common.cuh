// Shared host/device helpers of libvesper_b200: status codes, the thread-local error message,
// element-type dispatch and vector loads. Every kernel of the library is written for sm_100a.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "vesper_b200.h"

namespace vb {

// Records the message returned by vb_last_error() for the calling host thread.
void set_error(const char* fmt, ...);
void clear_error();
// Counts kernel launches made by this library (read with vb_launch_count()).
void count_launch();

#define VB_REQUIRE(cond, ...)                \
  do {                                       \
    if (!(cond)) {                           \
      ::vb::set_error(__VA_ARGS__);          \
      return VB_ERR_INVALID;                 \
    }                                        \
  } while (0)

#define VB_LAUNCH_CHECK(what)                                                        \
  do {                                                                               \
    cudaError_t e_ = cudaGetLastError();                                             \
    if (e_ != cudaSuccess) {                                                         \
      ::vb::set_error("%s: launch failed: %s", what, cudaGetErrorString(e_));        \
      return VB_ERR_CUDA;                                                            \
    }                                                                                \
    ::vb::count_launch();                                                            \
  } while (0)

#define VB_CUDA_CHECK(call, what)                                                    \
  do {                                                                               \
    cudaError_t e_ = (call);                                                         \
    if (e_ != cudaSuccess) {                                                         \
      ::vb::set_error("%s: %s", what, cudaGetErrorString(e_));                       \
      return VB_ERR_CUDA;                                                            \
    }                                                                                \
  } while (0)

inline int dtype_size(int dtype) {
  return dtype == VB_F32 ? 4 : (dtype == VB_BF16 || dtype == VB_F16) ? 2 : 0;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- element conversion -------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Loads N consecutive elements (N * sizeof(T) a multiple of 16 bytes when vec is true) as floats.
template <typename T, int N>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&out)[N]) {
  static_assert((N * sizeof(T)) % 16 == 0, "vector load must be whole 16-byte words");
  constexpr int WORDS = N * sizeof(T) / 16;
#pragma unroll
  for (int w = 0; w < WORDS; ++w) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(p) + w);
    const T* e = reinterpret_cast<const T*>(&raw);
    constexpr int PER = 16 / sizeof(T);
#pragma unroll
    for (int i = 0; i < PER; ++i) out[w * PER + i] = to_f32<T>(e[i]);
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_vec(T* __restrict__ p, const float (&in)[N]) {
  static_assert((N * sizeof(T)) % 16 == 0, "vector store must be whole 16-byte words");
  constexpr int WORDS = N * sizeof(T) / 16;
  constexpr int PER = 16 / sizeof(T);
#pragma unroll
  for (int w = 0; w < WORDS; ++w) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < PER; ++i) e[i] = from_f32<T>(in[w * PER + i]);
    reinterpret_cast<uint4*>(p)[w] = raw;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Dispatches a templated launcher on the runtime element type code.
#define VB_DISPATCH_DTYPE(code, T, ...)                    \
  [&]() -> int {                                           \
    switch (code) {                                        \
      case VB_F32: { using T = float; return __VA_ARGS__(); }          \
      case VB_BF16: { using T = __nv_bfloat16; return __VA_ARGS__(); } \
      case VB_F16: { using T = __half; return __VA_ARGS__(); }         \
      default: ::vb::set_error("unsupported dtype code %d", (int)(code)); return VB_ERR_INVALID; \
    }                                                      \
  }()

}  // namespace vb
