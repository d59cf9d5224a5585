// SwiGLU between the grouped GEMMs: h = silu(gate) * up, and its backward.
//
// The reference computes it as two PyTorch elementwise passes, `F.silu(gate) * up`
// (tests/test_moe.py:82), whose autograd backward adds three more.  One kernel each way
// here (16-byte vectors, grid-stride), with the same rounding sequence as those passes:
//   forward   s = rnd(silu(g)), h = rnd(s * u)                      (silu in fp32)
//   backward  du = rnd(dh * s), ds = rnd(dh * u),
//             dg = rnd(ds * sig(g) * (1 + g * (1 - sig(g))))        (fp32, sig = sigmoid)
// where rnd rounds fp32 to the tensor dtype.  Bytes per element: forward 2 reads + 1 write,
// backward 3 reads + 2 writes.
#pragma once

#include "common.cuh"

namespace moe {

template <typename T>
__device__ __forceinline__ float rnd(float v) { return to_f32(from_f32<T>(v)); }

// Logistic function in fp32 (expf and an IEEE division); every kernel that applies the
// SwiGLU uses this one definition.
__device__ __forceinline__ float sigmoid_f32(float x) { return 1.f / (1.f + expf(-x)); }

template <typename T>
__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const T* __restrict__ g, const T* __restrict__ u,
                                                         T* __restrict__ h, int64_t n) {
  constexpr int V = 16 / sizeof(T);
  const int64_t nv = n / V;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += stride) {
    const uint4 gv = reinterpret_cast<const uint4*>(g)[i];
    const uint4 uv = reinterpret_cast<const uint4*>(u)[i];
    const T* gp = reinterpret_cast<const T*>(&gv);
    const T* up = reinterpret_cast<const T*>(&uv);
    uint4 hv;
    T* hp = reinterpret_cast<T*>(&hv);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float x = to_f32(gp[j]);
      const float s = rnd<T>(x * sigmoid_f32(x));
      hp[j] = from_f32<T>(s * to_f32(up[j]));
    }
    reinterpret_cast<uint4*>(h)[i] = hv;
  }
  // tail (n not a multiple of the vector width)
  for (int64_t i = nv * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float x = to_f32(g[i]);
    h[i] = from_f32<T>(rnd<T>(x * sigmoid_f32(x)) * to_f32(u[i]));
  }
}

// Backward of one element: d = upstream gradient, x = gate, uu = up (all as stored,
// widened to fp32); returns the unrounded fp32 gradients of gate and up.
template <typename T>
__device__ __forceinline__ void swiglu_bwd_elem(float d, float x, float uu, float& dgo, float& duo) {
  const float sg = sigmoid_f32(x);
  const float s = rnd<T>(x * sg);
  duo = d * s;
  const float ds = rnd<T>(d * uu);
  dgo = ds * (sg * (1.f + x * (1.f - sg)));
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const T* __restrict__ dh, const T* __restrict__ g,
                                                         const T* __restrict__ u, T* __restrict__ dg,
                                                         T* __restrict__ du, int64_t n) {
  constexpr int V = 16 / sizeof(T);
  const int64_t nv = n / V;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += stride) {
    const uint4 dv = reinterpret_cast<const uint4*>(dh)[i];
    const uint4 gv = reinterpret_cast<const uint4*>(g)[i];
    const uint4 uv = reinterpret_cast<const uint4*>(u)[i];
    const T* dp = reinterpret_cast<const T*>(&dv);
    const T* gp = reinterpret_cast<const T*>(&gv);
    const T* up = reinterpret_cast<const T*>(&uv);
    uint4 gov, uov;
    T* gop = reinterpret_cast<T*>(&gov);
    T* uop = reinterpret_cast<T*>(&uov);
#pragma unroll
    for (int j = 0; j < V; ++j) {
      float a, b;
      swiglu_bwd_elem<T>(to_f32(dp[j]), to_f32(gp[j]), to_f32(up[j]), a, b);
      gop[j] = from_f32<T>(a);
      uop[j] = from_f32<T>(b);
    }
    reinterpret_cast<uint4*>(dg)[i] = gov;
    reinterpret_cast<uint4*>(du)[i] = uov;
  }
  for (int64_t i = nv * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float a, b;
    swiglu_bwd_elem<T>(to_f32(dh[i]), to_f32(g[i]), to_f32(u[i]), a, b);
    dg[i] = from_f32<T>(a);
    du[i] = from_f32<T>(b);
  }
}

}  // namespace moe
