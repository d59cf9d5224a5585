// Counting-sort permute, unpermute (forward/backward) and permute_backward.
//
// Reference semantics (echogujy/moe_ops, triton_gmm_ops):
//   offsets / histogram   permute_ops.py:17-43   (offsets[E+1], offsets[0] = 0)
//   permute scatter       permute_ops.py:50-110  (row_id_map[k*T+t] = destination row)
//   unpermute forward     unpermute_ops.py:20-72
//   unpermute backward    unpermute_ops.py:93-172
//   permute backward      permute_ops.py:130-133 (= unpermute with prob = 1)
//
// The reference assigns destinations with one atomic per slot, so the order inside an
// expert group is whatever the GPU scheduler produced.  Here the order is fixed: slot
// j = t*K + k goes to  offsets[e] + #{ j' < j : expert(j') = e },  i.e. the order of a
// stable argsort of the flattened indices (the reference's own PyTorch oracle,
// tests/test_permute.py:16-37).  Four launches:
//   1. permute_hist_kernel   per-tile expert histogram  -> cnt[e][tile]
//   2. permute_scan_kernel   one block: exclusive scan of cnt in (e, tile) order, offsets
//   3. permute_rank_kernel   per-tile stable rank (warp match + per-warp column scan)
//                            -> row_id_map
//   4. permute_copy_kernel   token-major row copy: read input[t] once, write its K rows
//                            with 16-byte vector stores.
#pragma once

#include "common.cuh"

namespace moe {

constexpr int kPermTileWarps = 16;
constexpr int kPermTile = kPermTileWarps * 32;  // slots per tile
constexpr int kMaxExperts = 1024;

inline int64_t permute_num_tiles(int64_t num_slots) {
  return (num_slots + kPermTile - 1) / kPermTile;
}

// ---------------------------------------------------------------- 1. histogram
__global__ void __launch_bounds__(kPermTile)
permute_hist_kernel(const int32_t* __restrict__ flat, int64_t num_slots, int E,
                    int32_t* __restrict__ cnt, int64_t num_tiles) {
  extern __shared__ int32_t s_hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_hist[e] = 0;
  __syncthreads();
  const int64_t j = (int64_t)blockIdx.x * kPermTile + threadIdx.x;
  if (j < num_slots) {
    const int e = flat[j];
    if (e >= 0 && e < E) atomicAdd(&s_hist[e], 1);
    else raise_device_error(2);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[(int64_t)e * num_tiles + blockIdx.x] = s_hist[e];
}

// ---------------------------------------------------------------- 2. scan (single block)
// In place: cnt[e][tile] becomes the first destination row of expert e's slots in that
// tile; offsets[e] = first row of expert e, offsets[E] = number of valid slots.
constexpr int kScanThreads = 1024;
__global__ void __launch_bounds__(kScanThreads)
permute_scan_kernel(int32_t* __restrict__ cnt, int64_t num_tiles, int E,
                    int32_t* __restrict__ offsets) {
  __shared__ int32_t s_part[kScanThreads];
  const int64_t n = num_tiles * E;
  const int64_t chunk = (n + kScanThreads - 1) / kScanThreads;
  const int64_t lo = threadIdx.x * chunk;
  const int64_t hi = lo + chunk < n ? lo + chunk : n;
  int32_t sum = 0;
  for (int64_t i = lo; i < hi; ++i) sum += cnt[i];
  s_part[threadIdx.x] = sum;
  __syncthreads();
  // Hillis-Steele inclusive scan of the per-thread sums.
  for (int off = 1; off < kScanThreads; off <<= 1) {
    const int32_t v = threadIdx.x >= off ? s_part[threadIdx.x - off] : 0;
    __syncthreads();
    s_part[threadIdx.x] += v;
    __syncthreads();
  }
  int32_t run = s_part[threadIdx.x] - sum;  // exclusive prefix of this chunk
  for (int64_t i = lo; i < hi; ++i) {
    const int32_t c = cnt[i];
    cnt[i] = run;
    if (i % num_tiles == 0) offsets[i / num_tiles] = run;
    run += c;
  }
  if (threadIdx.x == kScanThreads - 1) offsets[E] = s_part[kScanThreads - 1];
}

// ---------------------------------------------------------------- 3. stable rank
__global__ void __launch_bounds__(kPermTile)
permute_rank_kernel(const int32_t* __restrict__ flat, int64_t num_slots, int64_t num_tokens,
                    int K, int E, const int32_t* __restrict__ base, int64_t num_tiles,
                    int32_t* __restrict__ row_id_map) {
  extern __shared__ int32_t s_cnt[];  // [kPermTileWarps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kPermTileWarps * E; i += blockDim.x) s_cnt[i] = 0;
  __syncthreads();
  const int64_t j = (int64_t)blockIdx.x * kPermTile + threadIdx.x;
  int e = -1;
  if (j < num_slots) {
    e = flat[j];
    if (e < 0 || e >= E) e = -1;
  }
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int intra = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && intra == 0) s_cnt[warp * E + e] = __popc(peers);
  __syncthreads();
  // Column scan over the warps of this tile, seeded with the tile's global base.
  for (int x = threadIdx.x; x < E; x += blockDim.x) {
    int32_t run = base[(int64_t)x * num_tiles + blockIdx.x];
#pragma unroll
    for (int w = 0; w < kPermTileWarps; ++w) {
      const int32_t c = s_cnt[w * E + x];
      s_cnt[w * E + x] = run;
      run += c;
    }
  }
  __syncthreads();
  if (j < num_slots) {
    const int64_t t = j / K, k = j - t * K;
    row_id_map[k * num_tokens + t] = e >= 0 ? s_cnt[warp * E + e] + intra : -1;
  }
}

// ---------------------------------------------------------------- vector helpers
// 16-byte vector of 8 16-bit or 4 32-bit elements.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = to_f32(h[i]);
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack16(const float* f) {
  uint4 u;
  if constexpr (sizeof(T) == 4) {
    u.x = __float_as_uint(f[0]); u.y = __float_as_uint(f[1]);
    u.z = __float_as_uint(f[2]); u.w = __float_as_uint(f[3]);
  } else {
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = from_f32<T>(f[i]);
  }
  return u;
}

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

constexpr int kRowWarps = 8;  // warps (tokens) per block for the row kernels

// ---------------------------------------------------------------- 4. copy (token-major)
// VEC: rows are 16-byte multiples and 16-byte aligned (uint4 path), else element path.
template <typename T, bool VEC>
__global__ void __launch_bounds__(kRowWarps * 32)
permute_copy_kernel(const T* __restrict__ input, const int32_t* __restrict__ row_id_map,
                    T* __restrict__ permuted, int64_t num_tokens, int K, int64_t num_cols) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  int32_t dst_lane = -1;
  if (lane < K) dst_lane = row_id_map[(int64_t)lane * num_tokens + t];
  const T* src = input + t * num_cols;
  if constexpr (VEC) {
    const int64_t nv = num_cols / Vec16<T>::N;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    constexpr int U = 4;
    for (int64_t c0 = 0; c0 < nv; c0 += 32 * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + u * 32 + lane;
        if (c < nv) v[u] = ld_stream(s4 + c);
      }
      for (int k = 0; k < K; ++k) {
        const int32_t d = __shfl_sync(0xffffffffu, dst_lane, k);
        if (d < 0) continue;
        uint4* d4 = reinterpret_cast<uint4*>(permuted + (int64_t)d * num_cols);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t c = c0 + u * 32 + lane;
          if (c < nv) d4[c] = v[u];
        }
      }
    }
  } else {
    // Warp-uniform loop: every lane takes part in the shuffles.
    for (int64_t c0 = 0; c0 < num_cols; c0 += 32) {
      const int64_t c = c0 + lane;
      const bool in = c < num_cols;
      const T v = in ? src[c] : T();
      for (int k = 0; k < K; ++k) {
        const int32_t d = __shfl_sync(0xffffffffu, dst_lane, k);
        if (in && d >= 0) permuted[(int64_t)d * num_cols + c] = v;
      }
    }
  }
}

// ---------------------------------------------------------------- unpermute forward
// out[t] = sum_k p[t,k] * in[row_id_map[k*T+t]]; p == nullptr means p = 1.
// Accumulation: acc = 0; acc = rn(acc + rn(v * p)) for k = 0..K-1 (no FMA contraction),
// which is the rounding sequence of the reference's PyTorch oracle
// (tests/test_unpermute.py:25-35).  A slot with row -1 contributes nothing.
template <typename T, typename P, bool VEC>
__global__ void __launch_bounds__(kRowWarps * 32)
unpermute_fwd_kernel(const T* __restrict__ input, const int32_t* __restrict__ row_id_map,
                     const P* __restrict__ prob, T* __restrict__ out, int64_t num_tokens, int K,
                     int64_t num_cols) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  int32_t src_lane = -1;
  float p_lane = 1.f;
  if (lane < K) {
    src_lane = row_id_map[(int64_t)lane * num_tokens + t];
    if (prob != nullptr) p_lane = to_f32(prob[t * K + lane]);
  }
  T* dst = out + t * num_cols;
  if constexpr (VEC) {
    constexpr int NV = Vec16<T>::N;
    const int64_t nv = num_cols / NV;
    constexpr int U = 2;
    for (int64_t c0 = 0; c0 < nv; c0 += 32 * U) {
      float acc[U][NV];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int i = 0; i < NV; ++i) acc[u][i] = 0.f;
      for (int k = 0; k < K; ++k) {
        const int32_t s = __shfl_sync(0xffffffffu, src_lane, k);
        const float p = __shfl_sync(0xffffffffu, p_lane, k);
        if (s < 0) continue;
        const uint4* s4 = reinterpret_cast<const uint4*>(input + (int64_t)s * num_cols);
        uint4 raw[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t c = c0 + u * 32 + lane;
          if (c < nv) raw[u] = ld_stream(s4 + c);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          float f[NV];
          unpack16<T>(raw[u], f);
#pragma unroll
          for (int i = 0; i < NV; ++i) acc[u][i] = __fadd_rn(acc[u][i], __fmul_rn(f[i], p));
        }
      }
      uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + u * 32 + lane;
        if (c < nv) d4[c] = pack16<T>(acc[u]);
      }
    }
  } else {
    for (int64_t c0 = 0; c0 < num_cols; c0 += 32) {
      const int64_t c = c0 + lane;
      const bool in = c < num_cols;
      float acc = 0.f;
      for (int k = 0; k < K; ++k) {
        const int32_t s = __shfl_sync(0xffffffffu, src_lane, k);
        const float p = __shfl_sync(0xffffffffu, p_lane, k);
        if (s < 0 || !in) continue;
        acc = __fadd_rn(acc, __fmul_rn(to_f32(input[(int64_t)s * num_cols + c]), p));
      }
      if (in) dst[c] = from_f32<T>(acc);
    }
  }
}

// ---------------------------------------------------------------- unpermute backward
// act_grad[i] = cast(rn(g[t] * p[t,k])), prob_grad[t,k] = sum_c g[t,c] * in[i,c] (fp32),
// i = row_id_map[k*T+t].  grad_out[t] is read once per column block and reused for all K
// slots.  KMAX is the compile-time bound on K (the per-slot dot products live in
// registers).
template <typename T, typename P, int KMAX, bool VEC>
__global__ void __launch_bounds__(kRowWarps * 32)
unpermute_bwd_kernel(const T* __restrict__ grad_out, const T* __restrict__ input,
                     const int32_t* __restrict__ row_id_map, const P* __restrict__ prob,
                     T* __restrict__ act_grad, P* __restrict__ prob_grad, int64_t num_tokens,
                     int K, int64_t num_cols) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  int32_t src_lane = -1;
  float p_lane = 0.f;
  if (lane < K) {
    src_lane = row_id_map[(int64_t)lane * num_tokens + t];
    p_lane = to_f32(prob[t * K + lane]);
  }
  float dot[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) dot[k] = 0.f;
  const T* g_row = grad_out + t * num_cols;
  // Slot rows and probabilities, broadcast once (K <= KMAX <= 32).
  int32_t src_k[KMAX];
  float p_k[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    src_k[k] = __shfl_sync(0xffffffffu, src_lane, k);
    p_k[k] = __shfl_sync(0xffffffffu, p_lane, k);
  }
  if constexpr (VEC) {
    constexpr int NV = Vec16<T>::N;
    const int64_t nv = num_cols / NV;
    for (int64_t c = lane; c < nv; c += 32) {
      float g[NV];
      unpack16<T>(ld_stream(reinterpret_cast<const uint4*>(g_row) + c), g);
#pragma unroll
      for (int k = 0; k < KMAX; ++k) {
        if (k >= K) break;
        const int32_t s = src_k[k];
        const float p = p_k[k];
        if (s < 0) continue;
        float v[NV];
        unpack16<T>(ld_stream(reinterpret_cast<const uint4*>(input + (int64_t)s * num_cols) + c), v);
        float ag[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          dot[k] = fmaf(g[i], v[i], dot[k]);
          ag[i] = __fmul_rn(g[i], p);
        }
        reinterpret_cast<uint4*>(act_grad + (int64_t)s * num_cols)[c] = pack16<T>(ag);
      }
    }
  } else {
    for (int64_t c = lane; c < num_cols; c += 32) {
      const float g = to_f32(g_row[c]);
#pragma unroll
      for (int k = 0; k < KMAX; ++k) {
        if (k >= K) break;
        const int32_t s = src_k[k];
        const float p = p_k[k];
        if (s < 0) continue;
        const float v = to_f32(input[(int64_t)s * num_cols + c]);
        dot[k] = fmaf(g, v, dot[k]);
        act_grad[(int64_t)s * num_cols + c] = from_f32<T>(__fmul_rn(g, p));
      }
    }
  }
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    if (k >= K) break;
    float d = dot[k];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
    if (lane == 0) prob_grad[t * K + k] = from_f32<P>(d);
  }
}

}  // namespace moe
