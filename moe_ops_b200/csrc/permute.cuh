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
// tests/test_permute.py:16-37).  Three launches:
//   1. permute_hist_kernel   per-tile expert histogram -> cnt[e][tile]
//   2. permute_rank_kernel   per tile: its bases from the whole (small) count matrix, the
//                            offsets (block 0), then the stable rank (warp match + per-warp
//                            column scan) -> row_id_map
//   3. permute_copy_kernel   token-major row copy: read input[t] once, write its K rows
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
  pdl_launch_dependents();
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

// ---------------------------------------------------------------- 2. bases + stable rank
// Each block derives what it needs from the whole count matrix cnt[E][num_tiles] (small,
// L2-resident), so no separate scan launch is needed:
//   base[e] = offsets[e] + sum_{t < tile} cnt[e][t],  offsets[e] = sum_{e' < e, all t} cnt.
// Block 0 also writes offsets[E+1].  Then the tile's slots are ranked stably: warp match for
// the rank inside a warp, a per-warp column scan across the warps of the tile.
//
// Capacity (dropping): a slot whose stable rank inside its expert is >= `capacity`, or
// whose destination row would be >= `row_limit`, is dropped: row_id_map = -1 and no row.
// The offsets count the kept rows only, so the grouped GEMMs never see a dropped slot.
// Both limits at INT32_MAX give the plain permute.  `row_src` (nullable) receives the
// inverse map: row_src[row] = the token whose slot lands in that row.
// Dynamic shared memory: (kPermTileWarps + 3) * E int32.
__global__ void __launch_bounds__(kPermTile)
permute_rank_kernel(const int32_t* __restrict__ flat, int64_t num_slots, int64_t num_tokens,
                    int K, int E, const int32_t* __restrict__ cnt, int64_t num_tiles,
                    int32_t* __restrict__ row_id_map, int32_t* __restrict__ offsets,
                    int32_t capacity, int32_t row_limit, int32_t* __restrict__ row_src) {
  pdl_launch_dependents();
  pdl_wait();  // the histogram counts
  extern __shared__ int32_t s_cnt[];     // [kPermTileWarps][E]
  int32_t* s_before = s_cnt + kPermTileWarps * E;  // [E] this expert's rows in earlier tiles
  int32_t* s_total = s_before + E;                 // [E] this expert's rows in all tiles
  int32_t* s_first = s_total + E;                  // [E] first output row of the expert
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile = blockIdx.x;
  for (int i = threadIdx.x; i < kPermTileWarps * E; i += blockDim.x) s_cnt[i] = 0;
  // Per-expert sums over the tiles (a warp per expert, lanes over tiles).
  for (int x = warp; x < E; x += kPermTileWarps) {
    int32_t before = 0, total = 0;
    for (int64_t t = lane; t < num_tiles; t += 32) {
      const int32_t c = cnt[(int64_t)x * num_tiles + t];
      total += c;
      if (t < tile) before += c;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      before += __shfl_xor_sync(0xffffffffu, before, off);
      total += __shfl_xor_sync(0xffffffffu, total, off);
    }
    if (lane == 0) { s_before[x] = before; s_total[x] = total; }
  }
  __syncthreads();
  // Exclusive prefix of the kept totals over experts (one warp; E <= kMaxExperts).
  if (warp == 0) {
    int32_t carry = 0;
    for (int x0 = 0; x0 < E; x0 += 32) {
      const int x = x0 + lane;
      const int32_t v = x < E ? min(s_total[x], capacity) : 0;
      int32_t inc = v;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int32_t o = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += o;
      }
      if (x < E) {
        const int32_t first = carry + inc - v;  // offsets[x] before the row limit
        if (tile == 0) offsets[x] = min(first, row_limit);
        s_first[x] = first;
      }
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (tile == 0 && lane == 0) offsets[E] = min(carry, row_limit);
  }
  const int64_t j = tile * kPermTile + threadIdx.x;
  int e = -1;
  if (j < num_slots) {
    e = flat[j];
    if (e < 0 || e >= E) e = -1;
  }
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int intra = __popc(peers & ((1u << lane) - 1u));
  __syncthreads();
  if (e >= 0 && intra == 0) s_cnt[warp * E + e] = __popc(peers);
  __syncthreads();
  for (int x = threadIdx.x; x < E; x += blockDim.x) {
    int32_t run = s_before[x];
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
    int32_t dst = -1;
    if (e >= 0) {
      const int32_t r = s_cnt[warp * E + e] + intra;  // stable rank inside expert e
      if (r < capacity && s_first[e] + r < row_limit) dst = s_first[e] + r;
    }
    row_id_map[k * num_tokens + t] = dst;
    if (row_src != nullptr && dst >= 0) row_src[dst] = (int32_t)t;  // inverse map: row -> token
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

// Where the K rows of token t live.  The row kernels below read a slot's (rank, row) in lane
// k, broadcast it with shuffles and turn it into a pointer with at().
//   LocalRows: one buffer, rows from row_id_map (k-major [K*T], -1 = no row).
//   PeerRows:  rows spread over the ranks' buffers (expert parallelism over peer memory):
//              slot j = k*T + t lives in bases[ranks[j]] at row rows[j]; ranks[j] < 0 = none.
//              When `status` is given and reads 0 (a cross-GPU barrier of this step gave
//              up), every slot reads as none: the kernel touches no peer buffer, because
//              the peers may still be using them.
template <typename T>
struct LocalRows {
  static constexpr bool kPeer = false;
  T* base;
  const int32_t* map;
  int64_t num_tokens, num_cols;
  __device__ __forceinline__ int32_t row(int k, int64_t t) const {
    return map[(int64_t)k * num_tokens + t];
  }
  __device__ __forceinline__ int32_t rank(int, int64_t) const { return 0; }
  __device__ __forceinline__ T* at(int32_t, int32_t r) const { return base + (int64_t)r * num_cols; }
};

template <typename T>
struct PeerRows {
  static constexpr bool kPeer = true;
  T* const* bases;
  const int32_t* ranks;
  const int32_t* rows;
  int64_t num_tokens, num_cols;
  const int32_t* status;  // nullable
  __device__ __forceinline__ int32_t row(int k, int64_t t) const {
    if (status != nullptr && *status == 0) return -1;
    const int64_t j = (int64_t)k * num_tokens + t;
    return ranks[j] < 0 ? -1 : rows[j];
  }
  __device__ __forceinline__ int32_t rank(int k, int64_t t) const {
    return ranks[(int64_t)k * num_tokens + t];
  }
  __device__ __forceinline__ T* at(int32_t rk, int32_t r) const {
    return bases[rk] + (int64_t)r * num_cols;
  }
};

// ---------------------------------------------------------------- 4. copy (token-major)
// 16-byte loads each lane keeps in flight in the row kernels (measured on B200, cfg3 rows of
// 8 KB, K = 2, against the HBM copy bandwidth): the permute copy holds 16 chunks of its
// token's row (71 % -> 75 % with the launch changes); the unpermute kernels issue the loads
// of all K slots of a column block before using the first (8 loads: forward 79 % -> 94 %;
// 16 loads with the output-gradient chunks: backward 79 % -> 89.5 %).
#ifndef MOE_PERMUTE_COPY_U
#define MOE_PERMUTE_COPY_U 16
#endif
#ifndef MOE_UNPERMUTE_LOADS
#define MOE_UNPERMUTE_LOADS 8
#endif
#ifndef MOE_UNPERMUTE_BWD_LOADS
#define MOE_UNPERMUTE_BWD_LOADS 16
#endif
// VEC: rows are 16-byte multiples and 16-byte aligned (uint4 path), else element path.
template <typename T, bool VEC, class Rows>
__global__ void __launch_bounds__(kRowWarps * 32)
permute_copy_kernel(const T* __restrict__ input, Rows dst_rows, int64_t num_tokens, int K,
                    int64_t num_cols) {
  pdl_wait();  // row_id_map
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  int32_t dst_lane = -1, rank_lane = 0;
  if (lane < K) {
    dst_lane = dst_rows.row(lane, t);
    if constexpr (Rows::kPeer) rank_lane = dst_rows.rank(lane, t);
  }
  const T* src = input + t * num_cols;
  if constexpr (VEC) {
    const int64_t nv = num_cols / Vec16<T>::N;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    // U 16-byte chunks per lane in flight: a warp holds U * 512 bytes of its row.
    constexpr int U = MOE_PERMUTE_COPY_U;
    for (int64_t c0 = 0; c0 < nv; c0 += 32 * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + u * 32 + lane;
        if (c < nv) v[u] = ld_stream(s4 + c);
      }
      for (int k = 0; k < K; ++k) {
        const int32_t d = __shfl_sync(0xffffffffu, dst_lane, k);
        const int32_t rk = Rows::kPeer ? __shfl_sync(0xffffffffu, rank_lane, k) : 0;
        if (d < 0) continue;
        uint4* d4 = reinterpret_cast<uint4*>(dst_rows.at(rk, d));
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
        const int32_t rk = Rows::kPeer ? __shfl_sync(0xffffffffu, rank_lane, k) : 0;
        if (in && d >= 0) dst_rows.at(rk, d)[c] = v;
      }
    }
  }
}

// ---------------------------------------------------------------- unpermute forward
// out[t] = sum_k p[t,k] * in[row_id_map[k*T+t]]; p == nullptr means p = 1.
// Accumulation: acc = 0; acc = rn(acc + rn(v * p)) for k = 0..K-1 (no FMA contraction),
// which is the rounding sequence of the reference's PyTorch oracle
// (tests/test_unpermute.py:25-35).  A slot with row -1 contributes nothing.
// KMAX >= K: the K slots' loads of a column block are all issued before the first is used
// (KMAX * U 16-byte loads in flight per lane), then summed in k order.
template <typename T, typename P, int KMAX, bool VEC, class Rows>
__global__ void __launch_bounds__(kRowWarps * 32)
unpermute_fwd_kernel(Rows src_rows, const P* __restrict__ prob, T* __restrict__ out,
                     int64_t num_tokens, int K, int64_t num_cols) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  int32_t src_lane = -1, rank_lane = 0;
  float p_lane = 1.f;
  if (lane < K) {
    src_lane = src_rows.row(lane, t);
    if constexpr (Rows::kPeer) rank_lane = src_rows.rank(lane, t);
    if (prob != nullptr) p_lane = to_f32(prob[t * K + lane]);
  }
  T* dst = out + t * num_cols;
  if constexpr (VEC) {
    constexpr int NV = Vec16<T>::N;
    const int64_t nv = num_cols / NV;
    constexpr int U = KMAX >= MOE_UNPERMUTE_LOADS ? 1 : MOE_UNPERMUTE_LOADS / KMAX;
    int32_t s_k[KMAX];
    int32_t rk_k[KMAX];
    float p_k[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      s_k[k] = __shfl_sync(0xffffffffu, src_lane, k);
      rk_k[k] = Rows::kPeer ? __shfl_sync(0xffffffffu, rank_lane, k) : 0;
      p_k[k] = __shfl_sync(0xffffffffu, p_lane, k);
      if (k >= K) s_k[k] = -1;
    }
    for (int64_t c0 = 0; c0 < nv; c0 += 32 * U) {
      uint4 raw[KMAX][U];
#pragma unroll
      for (int k = 0; k < KMAX; ++k) {
        if (s_k[k] < 0) continue;
        const uint4* s4 = reinterpret_cast<const uint4*>(src_rows.at(rk_k[k], s_k[k]));
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t c = c0 + u * 32 + lane;
          if (c < nv) raw[k][u] = ld_stream(s4 + c);
        }
      }
      float acc[U][NV];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int i = 0; i < NV; ++i) acc[u][i] = 0.f;
#pragma unroll
      for (int k = 0; k < KMAX; ++k) {
        if (s_k[k] < 0) continue;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          float f[NV];
          unpack16<T>(raw[k][u], f);
#pragma unroll
          for (int i = 0; i < NV; ++i) acc[u][i] = __fadd_rn(acc[u][i], __fmul_rn(f[i], p_k[k]));
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
        const int32_t rk = Rows::kPeer ? __shfl_sync(0xffffffffu, rank_lane, k) : 0;
        const float p = __shfl_sync(0xffffffffu, p_lane, k);
        if (s < 0 || !in) continue;
        acc = __fadd_rn(acc, __fmul_rn(to_f32(src_rows.at(rk, s)[c]), p));
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
// in_rows and act_rows share one slot map (the same rank and row for each slot); they differ
// in the buffers they point into.
template <typename T, typename P, int KMAX, bool VEC, class RowsIn, class RowsOut>
__global__ void __launch_bounds__(kRowWarps * 32)
unpermute_bwd_kernel(const T* __restrict__ grad_out, RowsIn in_rows, RowsOut act_rows,
                     const P* __restrict__ prob, P* __restrict__ prob_grad, int64_t num_tokens,
                     int K, int64_t num_cols) {
  static_assert(RowsIn::kPeer == RowsOut::kPeer, "one slot map for both row sets");
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRowWarps + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  int32_t src_lane = -1, rank_lane = 0;
  float p_lane = 0.f;
  if (lane < K) {
    src_lane = in_rows.row(lane, t);
    if constexpr (RowsIn::kPeer) rank_lane = in_rows.rank(lane, t);
    p_lane = to_f32(prob[t * K + lane]);
  }
  float dot[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) dot[k] = 0.f;
  const T* g_row = grad_out + t * num_cols;
  // Slot rows and probabilities, broadcast once (K <= KMAX <= 32).
  int32_t src_k[KMAX];
  int32_t rank_k[RowsIn::kPeer ? KMAX : 1];
  float p_k[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    src_k[k] = __shfl_sync(0xffffffffu, src_lane, k);
    if constexpr (RowsIn::kPeer) rank_k[k] = __shfl_sync(0xffffffffu, rank_lane, k);
    p_k[k] = __shfl_sync(0xffffffffu, p_lane, k);
  }
  if constexpr (VEC) {
    // U 16-byte chunks per lane and iteration: all their loads are issued before use.
    constexpr int NV = Vec16<T>::N;
    constexpr int U = KMAX >= MOE_UNPERMUTE_BWD_LOADS ? 1 : MOE_UNPERMUTE_BWD_LOADS / KMAX;
    const int64_t nv = num_cols / NV;
    for (int64_t c0 = 0; c0 < nv; c0 += 32 * U) {
      uint4 graw[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t c = c0 + u * 32 + lane;
        if (c < nv) graw[u] = ld_stream(reinterpret_cast<const uint4*>(g_row) + c);
      }
      // every slot's rows of this column block in flight before the first is used
      uint4 vraw[KMAX][U];
#pragma unroll
      for (int k = 0; k < KMAX; ++k) {
        if (k >= K || src_k[k] < 0) continue;
        const int32_t rk = RowsIn::kPeer ? rank_k[RowsIn::kPeer ? k : 0] : 0;
        const uint4* in4 = reinterpret_cast<const uint4*>(in_rows.at(rk, src_k[k]));
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t c = c0 + u * 32 + lane;
          if (c < nv) vraw[k][u] = ld_stream(in4 + c);
        }
      }
#pragma unroll
      for (int k = 0; k < KMAX; ++k) {
        if (k >= K) break;
        const int32_t s = src_k[k];
        const float p = p_k[k];
        if (s < 0) continue;
        const int32_t rk = RowsIn::kPeer ? rank_k[RowsIn::kPeer ? k : 0] : 0;
        uint4* ag4 = reinterpret_cast<uint4*>(act_rows.at(rk, s));
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int64_t c = c0 + u * 32 + lane;
          if (c >= nv) continue;
          float g[NV], v[NV], ag[NV];
          unpack16<T>(graw[u], g);
          unpack16<T>(vraw[k][u], v);
#pragma unroll
          for (int i = 0; i < NV; ++i) {
            dot[k] = fmaf(g[i], v[i], dot[k]);
            ag[i] = __fmul_rn(g[i], p);
          }
          ag4[c] = pack16<T>(ag);
        }
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
        const int32_t rk = RowsIn::kPeer ? rank_k[RowsIn::kPeer ? k : 0] : 0;
        const float v = to_f32(in_rows.at(rk, s)[c]);
        dot[k] = fmaf(g, v, dot[k]);
        act_rows.at(rk, s)[c] = from_f32<T>(__fmul_rn(g, p));
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
