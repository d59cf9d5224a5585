// Expert parallelism over peer memory: the kernels that let dispatch and combine move rows
// straight between the GPUs' buffers over NVLink instead of through an all-to-all.
//
// The reference has no multi-GPU path.  This is the dispatch/combine of an expert-parallel
// MoE layer: rank r owns experts [r*El, (r+1)*El); every rank keeps its own tokens.
//
// Layout.  Each rank's receive buffer holds the rows it computes on, grouped by local
// expert and, inside an expert, by source rank: the grouped GEMM's layout, so no regroup
// pass is needed.  A slot (t, k) of this rank's tokens whose expert is e goes to rank
// e / El at row  row_id_map[k*T+t] + delta[e],  where row_id_map is this rank's stable
// counting-sort position (the permute's index pass) and delta[e] moves expert e's block of
// this rank's rows to where the owner expects it (computed from all ranks' counts).
//
// The row kernels themselves are the permute / unpermute kernels of permute.cuh run with
// PeerRows, whose rows live in the buffers named by a table of per-rank base pointers
// (this rank's own buffer and the peers' buffers opened through CUDA IPC).
//
// The barrier signals every peer, then waits for every peer's signal, with a time limit.
#pragma once

#include "common.cuh"
#include "sm100_ptx.cuh"

namespace moe {

// ranks[j] / rows[j] of slot j = k*T + t.  A slot whose expert or destination row is out of
// range gets rank -1 (the row kernels skip it) and raises device error 3: no kernel ever
// stores outside a receive buffer.
__global__ void __launch_bounds__(256)
ep_slot_map_kernel(const int32_t* __restrict__ indices, const int32_t* __restrict__ row_id_map,
                   const int32_t* __restrict__ delta, int64_t num_tokens, int K, int E,
                   int experts_per_rank, int world, int64_t capacity, int32_t* __restrict__ ranks,
                   int32_t* __restrict__ rows) {
  const int64_t n = num_tokens * K;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = j / num_tokens, t = j - k * num_tokens;
    const int e = indices[t * K + k];
    int32_t rank = -1, row = 0;
    if (e >= 0 && e < E) {
      const int r = e / experts_per_rank;
      const int64_t dst = (int64_t)row_id_map[j] + delta[e];
      if (r < world && dst >= 0 && dst < capacity) {
        rank = r;
        row = (int32_t)dst;
      }
    }
    if (rank < 0) raise_device_error(3);
    ranks[j] = rank;
    rows[j] = row;
  }
}

// One warp.  The barrier's epoch is this rank's device counter plus one (written back at the
// end), so a launch captured in a CUDA graph advances it on every replay.  Lane i < world:
// make this rank's earlier writes visible system-wide, then store the epoch into slot `me`
// of rank i's flag array (a peer store over NVLink, or a local one for i == me).  Then lane
// i waits until slot i of this rank's own array reaches the epoch, giving up after
// timeout_ns (device error 4, *status = 0; a barrier that completes leaves *status as it
// was, so a failure stays visible).  Epochs increase by one per barrier on every rank, so
// a flag never needs resetting.
__global__ void ep_barrier_kernel(int64_t* const* __restrict__ flags, int me, int world,
                                  int64_t* __restrict__ epoch_counter, uint64_t timeout_ns,
                                  int32_t* __restrict__ status) {
  const int lane = threadIdx.x;
  const int64_t epoch = *epoch_counter + 1;
  __threadfence_system();
  if (lane < world) {
    int64_t* slot = flags[lane] + me;
    asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(slot), "l"(epoch) : "memory");
  }
  bool ok = true;
  if (lane < world) {
    const int64_t* mine = flags[me] + lane;
    const uint64_t t0 = ptx::globaltimer();
    for (uint32_t it = 0;; ++it) {
      int64_t v;
      asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(mine) : "memory");
      if (v >= epoch) break;
      if ((it & 255u) == 255u && ptx::globaltimer() - t0 > timeout_ns) {
        ok = false;
        break;
      }
    }
  }
  const bool all_ok = __all_sync(0xffffffffu, ok);
  if (lane == 0) {
    *epoch_counter = epoch;
    if (!all_ok) {
      raise_device_error(4);
      if (status != nullptr) *status = 0;
    }
  }
  __threadfence_system();
}

// Counts exchange for the peer-memory layout: this rank's [E] counts go to row `me` of
// every rank's [world, E] array (peer stores; the barrier that follows makes them visible).
__global__ void __launch_bounds__(256)
ep_put_counts_kernel(const int32_t* __restrict__ counts, int E, int32_t* const* __restrict__ dst,
                     int me, int world) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < E * world; i += gridDim.x * blockDim.x) {
    const int r = i / E, e = i - r * E;
    dst[r][(int64_t)me * E + e] = counts[e];
  }
}

// dst[r] = rnd(dst[r] + src[r]) for the first min(*n_rows, max_rows) rows (fp32 sum rounded
// to T, as a PyTorch add of two 16-bit tensors).  The row count stays on the device, so
// buffers sized for the worst case cost only their live rows.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
add_rows_kernel(T* __restrict__ dst, const T* __restrict__ src, const int32_t* __restrict__ n_rows,
                int64_t max_rows, int64_t cols) {
  const int64_t rows = min((int64_t)*n_rows, max_rows);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if constexpr (VEC) {
    constexpr int NV = 16 / sizeof(T);
    const int64_t n = rows * cols / NV;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
      uint4 a = reinterpret_cast<const uint4*>(dst)[i];
      const uint4 b = reinterpret_cast<const uint4*>(src)[i];
      T* pa = reinterpret_cast<T*>(&a);
      const T* pb = reinterpret_cast<const T*>(&b);
#pragma unroll
      for (int j = 0; j < NV; ++j) pa[j] = from_f32<T>(to_f32(pa[j]) + to_f32(pb[j]));
      reinterpret_cast<uint4*>(dst)[i] = a;
    }
  } else {
    const int64_t n = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
      dst[i] = from_f32<T>(to_f32(dst[i]) + to_f32(src[i]));
  }
}

}  // namespace moe
