// Fused top-k softmax (router) forward and backward: one warp per token.
//
// Semantics follow the reference's Triton kernels
//   forward  triton_gmm_ops/fused_topk_softmax_ops.py:17-70
//   backward triton_gmm_ops/fused_topk_softmax_ops.py:83-114
// Forward: K rounds of "take the largest remaining logit, lowest expert index on ties,
// then overwrite it with -inf"; a softmax over the K picked values in fp32; weights are
// written in the logits dtype and indices as int32.
// Backward: dlogit[t, idx[t,k]] = w*(g - sum_k g*w) (fp32, cast to the weights dtype),
// zero at every other expert.  The backward writes the whole [T, E] row itself, so no
// separate memset of grad_logits is needed.
#pragma once

#include "common.cuh"

namespace moe {

constexpr int kTopkWarpsPerBlock = 8;
#ifndef MOE_TOPK_BLOCKS_PER_SM
#define MOE_TOPK_BLOCKS_PER_SM 2
#endif

struct ArgBest {
  float v;
  int i;
};

// true if a ranks before b: larger value, or equal value and lower index.
__device__ __forceinline__ bool ranks_before(float av, int ai, float bv, int bi) {
  return av > bv || (av == bv && ai < bi);
}

// VPT = logits held per lane (E <= 32*VPT).
template <typename T, int VPT>
__global__ void __launch_bounds__(kTopkWarpsPerBlock * 32)
topk_softmax_fwd_kernel(const T* __restrict__ logits, T* __restrict__ weights,
                        int32_t* __restrict__ indices, int64_t num_tokens, int E, int K) {
  const int lane = threadIdx.x & 31;
  // Warps stride over the tokens (a grid of a few blocks per SM): fewer, longer-lived blocks
  // than one block per 8 tokens.
  const int64_t warps = (int64_t)gridDim.x * kTopkWarpsPerBlock;
  for (int64_t t = (int64_t)blockIdx.x * kTopkWarpsPerBlock + (threadIdx.x >> 5); t < num_tokens;
       t += warps) {
  const T* row = logits + t * E;

  float v[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = j * 32 + lane;
    v[j] = e < E ? to_f32(row[e]) : -INFINITY;
  }

  float my_val = -INFINITY;  // lane k keeps the k-th pick
  int my_idx = 0;
  for (int k = 0; k < K; ++k) {
    // Lane-local best: values are visited in increasing expert order, so a strict
    // comparison keeps the lowest index among equal values.
    float bv = v[0];
    int bi = lane;
#pragma unroll
    for (int j = 1; j < VPT; ++j) {
      const int e = j * 32 + lane;
      if (e < E && v[j] > bv) { bv = v[j]; bi = e; }
    }
    if (lane >= E) { bv = -INFINITY; bi = 0x7fffffff; }
    // Butterfly arg-max across the warp.
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ranks_before(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == k) { my_val = bv; my_idx = bi; }
    // The owner lane masks the winner with -inf (it may be picked again only through
    // an all -inf tie, exactly as in the reference).
    if ((bi & 31) == lane) {
#pragma unroll
      for (int j = 0; j < VPT; ++j)
        if (j == (bi >> 5)) v[j] = -INFINITY;
    }
  }

  // Softmax over the K picked values (fp32): max, exp, sum, divide.
  float m = my_val;
  if (lane >= K) m = -INFINITY;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  float ex = lane < K ? expf(my_val - m) : 0.f;
  float s = ex;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane < K) {
    weights[t * K + lane] = from_f32<T>(ex / s);
    indices[t * K + lane] = my_idx;
  }
  }  // token loop
}

// Small routers (E <= 8 * VPT, K <= 8): 8 lanes per token, 4 tokens per warp.  Same rule as
// above (largest remaining value, lowest index on ties, the winner masked with -inf), with
// 3-step butterflies inside each 8-lane group instead of 5-step ones across the warp: a
// quarter of the instructions per token.
template <typename T, int VPT>
__global__ void __launch_bounds__(kTopkWarpsPerBlock * 32)
topk_softmax_fwd_group8_kernel(const T* __restrict__ logits, T* __restrict__ weights,
                               int32_t* __restrict__ indices, int64_t num_tokens, int E, int K) {
  constexpr int G = 8;
  const int lane = threadIdx.x & 31;
  const int l = lane & (G - 1);
  const int64_t groups = (int64_t)gridDim.x * kTopkWarpsPerBlock * (32 / G);
  const int64_t first = ((int64_t)blockIdx.x * kTopkWarpsPerBlock + (threadIdx.x >> 5)) * (32 / G) +
                        (lane >> 3);
  // Every lane of the warp runs the same number of iterations (the shuffles need them all);
  // groups past the last token compute on -inf and store nothing.
  for (int64_t base = first - (lane >> 3); base < num_tokens; base += groups) {
    const int64_t t = base + (lane >> 3);
    const bool live = t < num_tokens;
    const T* row = logits + (live ? t : 0) * E;
    float v[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int e = j * G + l;
      v[j] = (live && e < E) ? to_f32(row[e]) : -INFINITY;
    }
    float my_val = -INFINITY;  // lane l of the group keeps the l-th pick
    int my_idx = 0;
    for (int k = 0; k < K; ++k) {
      float bv = v[0];
      int bi = l;
#pragma unroll
      for (int j = 1; j < VPT; ++j) {
        const int e = j * G + l;
        if (e < E && v[j] > bv) { bv = v[j]; bi = e; }
      }
      if (l >= E) { bv = -INFINITY; bi = 0x7fffffff; }
#pragma unroll
      for (int off = G / 2; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ranks_before(ov, oi, bv, bi)) { bv = ov; bi = oi; }
      }
      if (l == k) { my_val = bv; my_idx = bi; }
      if ((bi & (G - 1)) == l) {
#pragma unroll
        for (int j = 0; j < VPT; ++j)
          if (j == bi / G) v[j] = -INFINITY;
      }
    }
    float m = l < K ? my_val : -INFINITY;
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float ex = l < K ? expf(my_val - m) : 0.f;
    float s = ex;
#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (live && l < K) {
      weights[t * K + l] = from_f32<T>(ex / s);
      indices[t * K + l] = my_idx;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kTopkWarpsPerBlock * 32)
topk_softmax_bwd_kernel(const T* __restrict__ grad_w, const T* __restrict__ w,
                        const int32_t* __restrict__ idx, T* __restrict__ grad_logits,
                        int64_t num_tokens, int E, int K) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kTopkWarpsPerBlock + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  float g = 0.f, wv = 0.f;
  int e_k = -1;
  if (lane < K) {
    g = to_f32(grad_w[t * K + lane]);
    wv = to_f32(w[t * K + lane]);
    e_k = idx[t * K + lane];
  }
  float s = g * wv;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  const T dy = from_f32<T>(wv * (g - s));
  T* row = grad_logits + t * E;
  const T zero = from_f32<T>(0.f);
  for (int e = lane; e < E; e += 32) row[e] = zero;
  __syncwarp();
  if (lane < K && e_k >= 0 && e_k < E) row[e_k] = dy;
}

template <typename T>
int launch_topk_fwd(const void* logits, int64_t T_, int E, int K, void* weights, int32_t* indices,
                    cudaStream_t stream) {
  const int64_t blocks = (T_ + kTopkWarpsPerBlock - 1) / kTopkWarpsPerBlock;
  int dev = 0;
  cudaGetDevice(&dev);
  const int64_t cap = (int64_t)MOE_TOPK_BLOCKS_PER_SM * num_sms(dev);
  const dim3 grid((unsigned)(blocks < cap ? blocks : cap));
  const dim3 block(kTopkWarpsPerBlock * 32);
  const T* l = static_cast<const T*>(logits);
  T* w = static_cast<T*>(weights);
  if (E <= 64 && K <= 8) {
    // 4 tokens per warp: measured on B200 (T = 8192, E = 64, K = 2) against a warp per token
    const int64_t gblocks = (T_ + 4 * kTopkWarpsPerBlock - 1) / (4 * kTopkWarpsPerBlock);
    const dim3 ggrid((unsigned)(gblocks < cap ? gblocks : cap));
    if (E <= 32)
      topk_softmax_fwd_group8_kernel<T, 4><<<ggrid, block, 0, stream>>>(l, w, indices, T_, E, K);
    else
      topk_softmax_fwd_group8_kernel<T, 8><<<ggrid, block, 0, stream>>>(l, w, indices, T_, E, K);
    MOE_LAUNCH_CHECK();
    return MOE_OK;
  }
#define MOE_TOPK_CASE(VPT)                                                                   \
  if (E <= 32 * VPT) {                                                                       \
    topk_softmax_fwd_kernel<T, VPT><<<grid, block, 0, stream>>>(l, w, indices, T_, E, K);    \
    MOE_LAUNCH_CHECK();                                                                      \
    return MOE_OK;                                                                           \
  }
  MOE_TOPK_CASE(1)
  MOE_TOPK_CASE(2)
  MOE_TOPK_CASE(4)
  MOE_TOPK_CASE(8)
  MOE_TOPK_CASE(16)
  MOE_TOPK_CASE(32)
#undef MOE_TOPK_CASE
  return set_error(MOE_ERR_UNSUPPORTED, "topk_softmax: num_experts=%d > 1024", E);
}

template <typename T>
int launch_topk_bwd(const void* gw, const void* w, const int32_t* idx, int64_t T_, int E, int K,
                    void* grad_logits, cudaStream_t stream) {
  const dim3 grid((unsigned)((T_ + kTopkWarpsPerBlock - 1) / kTopkWarpsPerBlock));
  topk_softmax_bwd_kernel<T><<<grid, kTopkWarpsPerBlock * 32, 0, stream>>>(
      static_cast<const T*>(gw), static_cast<const T*>(w), idx, static_cast<T*>(grad_logits), T_,
      E, K);
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

}  // namespace moe
