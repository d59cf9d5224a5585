// Shared host/device helpers for the sm_100a MoE kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/moe_b200.h"

namespace moe {

// ------------------------------------------------------------------ host-side status
// Records a message for moe_last_error_string() and returns `code`.
int set_error(int code, const char* fmt, ...);

#define MOE_CUDA_CHECK(expr)                                                          \
  do {                                                                                \
    cudaError_t _e = (expr);                                                          \
    if (_e != cudaSuccess)                                                            \
      return ::moe::set_error(MOE_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,           \
                              cudaGetErrorString(_e), __FILE__, __LINE__);            \
  } while (0)

#define MOE_LAUNCH_CHECK()                                                            \
  do {                                                                                \
    cudaError_t _e = cudaGetLastError();                                              \
    if (_e != cudaSuccess)                                                            \
      return ::moe::set_error(MOE_ERR_CUDA, "kernel launch failed: %s (%s:%d)",       \
                              cudaGetErrorString(_e), __FILE__, __LINE__);            \
  } while (0)

#define MOE_REQUIRE(cond, ...)                                                        \
  do {                                                                                \
    if (!(cond)) return ::moe::set_error(MOE_ERR_INVALID_ARG, __VA_ARGS__);           \
  } while (0)

inline int dtype_size(int dtype) { return dtype == MOE_F32 ? 4 : 2; }
inline bool dtype_ok(int dtype) { return dtype == MOE_F32 || dtype == MOE_F16 || dtype == MOE_BF16; }

int num_sms(int device);

// ------------------------------------------------------------------ device error word
// Device-side error word shared by all kernels of the library (one per device; the
// library is built as a single translation unit, so this is its only definition).
// Codes: 1 = bounded wait gave up (GEMM pipeline), 2 = expert index out of range.
__device__ int g_device_error;

// Programmatic dependent launch: a kernel launched with programmatic stream serialization
// may start while the previous kernel of the stream still runs; pdl_wait() blocks until that
// kernel has completed and its memory is visible (a no-op for an ordinary launch).
// pdl_launch_dependents() lets the next kernel of the stream start early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void raise_device_error(int code) {
  atomicCAS(&g_device_error, 0, code);
}

// ------------------------------------------------------------------ element conversion
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f32(float v) { return v; }
  static __device__ __forceinline__ float from_f32(float v) { return v; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f32(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
};

template <typename T> __device__ __forceinline__ float to_f32(T v) { return Elem<T>::to_f32(v); }
template <typename T> __device__ __forceinline__ T from_f32(float v) { return Elem<T>::from_f32(v); }

// Dispatch a templated functor on a dtype code.
#define MOE_DISPATCH_DTYPE(code, T, ...)                                               \
  [&]() -> int {                                                                      \
    switch (code) {                                                                   \
      case MOE_F32: { using T = float; return __VA_ARGS__(); }                        \
      case MOE_F16: { using T = __half; return __VA_ARGS__(); }                       \
      case MOE_BF16: { using T = __nv_bfloat16; return __VA_ARGS__(); }               \
      default: return ::moe::set_error(MOE_ERR_INVALID_ARG, "bad dtype code %d", (int)(code)); \
    }                                                                                 \
  }()

}  // namespace moe
