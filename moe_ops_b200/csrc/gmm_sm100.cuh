// Persistent grouped GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the reference's grouped GEMM kernels
//   forward / dgrad  grouped_matmul_tma_kernel  triton_gmm_ops/grouped_gemm_ops_sm90.py:44-148
//                    gmm_forward_kernel         triton_gmm_ops/grouped_gemm_ops.py:20-69
//   wgrad            gmm_gradB_kernel           triton_gmm_ops/grouped_gemm_ops.py:126-165
//
// One kernel template, two modes:
//   kModeRows   (forward and dgrad): C[rows of g] = A[rows of g] . op(B[g]); the tiles of
//               expert g cover its ragged row range, the contraction length is fixed.
//               A is K-major; B[g] is K-major ([Nout, Kc]) or MN-major ([Kc, Nout]).
//   kModeWgrad  (wgrad): Out[g] = X[rows of g]^T . Y[rows of g]  ([P, Q] per expert); the
//               contraction runs over the ragged rows of expert g.  X and Y are MN-major.
//
// and two CTA-group shapes:
//   CG = 1  one CTA per tile, 128 x 256 tile, M=128 N=256 K=16 MMAs, 4 stages of 48 KB
//           (A in two 64-row boxes).
//   CG = 2  a cluster of two CTAs (an SM pair) per 256 x 256 tile running cta_group::2
//           MMAs (M=256, N=256): each CTA holds its own 128 rows of A and its own 128
//           columns of B, so each SM streams 32 KB instead of 48 KB per 64-deep k-block;
//           6 stages of 32 KB.  Only the pair's first CTA (the leader) issues MMAs.  Both
//           CTAs load with TMA into their own shared memory; the loads complete their
//           bytes on the leader's `full` barrier, which the leader alone arms with the
//           pair's byte count.  The leader's commits arrive on both CTAs' `empty` and
//           `tmem_full` barriers; both epilogues arrive on the leader's `tmem_empty` (the
//           peer with a relaxed remote arrive).  No cluster-scope fence sits on the hot
//           path: only a masked wgrad block hands its zeroed rows over with a
//           release/acquire pair (`peer_done`).  In kModeRows an expert's last tile of at
//           most 128 rows is a half tile: M=128 pair MMAs with 64 rows per CTA.
//           The host uses SM pairs for wgrad (P > 128) and single CTAs for kModeRows,
//           where they measured faster.
//
// Warp roles (384 threads, one CTA per SM, persistent over a static tile stride):
//   warp 0      TMA producer (one elected lane issues; it never waits on data).
//   warp 2      wgrad only: zero-fills the rows of masked blocks (see below).
//   warp 1      TMEM owner; in the MMA-issuing CTA one lane issues 4 tcgen05.mma per
//               stage into one of two TMEM accumulators (2 x 256 fp32 columns) and commits
//               each stage back to the producers.
//   warps 4-11  epilogue (8 warps, lane quarter = warp % 4, column half = (warp-4)/4):
//               tcgen05.ld, round to the output dtype, stage 32 x 32 blocks in a 2 KB
//               buffer laid out in the TMA 64-byte swizzle and write them with TMA stores
//               (or, for row tiles that end inside an expert, masked 64-byte row stores).
//               Releasing the accumulator lets the MMA warp start the tile after next, so
//               the epilogue overlaps the next tile's main loop.
//
// Ragged contraction (wgrad): the last 64-row block of an expert may reach into the next
// expert's rows.  The producer loads that block on the stage's `raw` barrier and moves on;
// the fix-up warp waits for it, zeroes the rows past the expert's end in shared memory,
// fences the generic->async proxy and then hands the stage to the MMA.
//
// Tile scheduler: each CTA builds the per-expert tile prefix from `offsets` in shared
// memory (no host sync), then the cluster walks tiles c, c + #clusters, ...  Inside an
// expert, tiles run row-block fastest so that concurrently running tiles share the same
// B tile through L2.  Empty experts own no tile in kModeRows; in kModeWgrad they own
// their full [P, Q] tiles, written as zeros.
//
// Every mbarrier wait is bounded (2 s); a wait that gives up sets a shared abort flag and
// the device error word, every role then leaves its loop and the TMEM is freed.
#pragma once

#include "common.cuh"
#include "sm100_ptx.cuh"
#include "swiglu.cuh"

#include <type_traits>

namespace moe {
namespace gmm {

constexpr int BN = 256;   // tile columns (both CTA-group shapes)
constexpr int BMC = 128;  // tile rows held by one CTA
constexpr int BK = 64;    // 64 x 16-bit = one 128-byte swizzle row
constexpr int UMMA_K = 16;
constexpr int kEpiWarps = 8;  // warps 4..11
constexpr int kThreads = 128 + 32 * kEpiWarps;
constexpr int kMaxGroups = 1024;
constexpr uint32_t kTmemCols = 2 * BN;
constexpr uint32_t kEpiBufBytes = 32 * 64;  // 32 rows x 32 16-bit columns (swizzled 16-B chunks)
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

#ifndef MOE_CG2_STAGES
#define MOE_CG2_STAGES 6
#endif
#ifndef MOE_CG2_EPI_BUFS
#define MOE_CG2_EPI_BUFS 1
#endif

template <int CG>
struct Shape {
  static constexpr int STAGES = CG == 1 ? 4 : MOE_CG2_STAGES;
  // Epilogue staging buffers per warp: a warp's next 32 x 32 block goes into the next
  // buffer while earlier TMA stores still read theirs.
  static constexpr int EPI_BUFS = CG == 1 ? 1 : MOE_CG2_EPI_BUFS;
  static constexpr int TILE_M = BMC * CG;                     // rows of the tile (pair)
  static constexpr int B_COLS = BN / CG;                      // B columns held by one CTA
  static constexpr uint32_t A_BYTES = BMC * BK * 2;           // per CTA per stage
  static constexpr uint32_t B_BYTES = B_COLS * BK * 2;        // per CTA per stage
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;  // per CTA per stage
};

enum Mode { kModeRows = 0, kModeWgrad = 1, kModeGateUp = 2, kModeSwiGLUBwd = 3 };

// Output columns one tile covers: a gate/up tile holds 128 gate and 128 up columns in its
// 256-column accumulator and writes 128 columns of each output.
template <int MODE>
__host__ __device__ constexpr int tile_out_cols() { return MODE == kModeGateUp ? BN / 2 : BN; }

template <int CG>
struct SmemLayout {
  uint8_t a[Shape<CG>::STAGES][Shape<CG>::A_BYTES];
  uint8_t b[Shape<CG>::STAGES][Shape<CG>::B_BYTES];
  uint8_t cbuf[kEpiWarps][Shape<CG>::EPI_BUFS][kEpiBufBytes];  // epilogue transpose buffers
  uint64_t full[Shape<CG>::STAGES];       // used in the leader CTA
  uint64_t empty[Shape<CG>::STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];                 // used in the leader CTA
  uint64_t raw[Shape<CG>::STAGES];        // masked wgrad block landed (before zeroing)
  uint64_t peer_done[Shape<CG>::STAGES];  // leader: the peer has zeroed its masked rows
  uint32_t tmem_base;
  int abort;
  int tile_prefix[kMaxGroups + 1];
  int warp_sums[kThreads / 32];
};
template <int CG>
constexpr size_t smem_bytes() { return sizeof(SmemLayout<CG>) + 1024; }  // + alignment slack

struct Params {
  const int32_t* offsets;
  int offsets_plus_one;  // 1: offsets has E+1 entries starting at 0; 0: E end offsets
  int num_groups;
  int64_t m_total;       // rows of A / X / Y
  int n_out;             // output columns (kModeRows: Nout, kModeWgrad: Q)
  int p_out;             // kModeWgrad: output rows per expert (P)
  int k_red;             // kModeRows: contraction length (Kc)
  void* out;             // kModeRows: C [m_total, n_out]; kModeWgrad: [E, p_out, n_out];
                         // kModeGateUp: h = silu(gate) * up [m_total, n_out]
  void* out_gate;        // kModeGateUp: gate = A . B_gate^T [m_total, n_out]
  void* out_up;          // kModeGateUp: up = A . B_up^T [m_total, n_out];
                         // kModeSwiGLUBwd: grad of up (`out` holds the grad of gate)
  const void* in_gate;   // kModeSwiGLUBwd: the forward's gate [m_total, n_out]
  const void* in_up;     // kModeSwiGLUBwd: the forward's up [m_total, n_out]
  int q_fastest;         // kModeWgrad: walk an expert's tiles output-column block fastest
  // Gathered operand (permute fused into the GEMM): row r of the operand is row
  // gather_rows[r] of a [gather_src_rows, ...] tensor, fetched with TMA gather4 (the map's
  // box is one row high).  Row mode (1-SM tiles): the operand is A; wgrad mode: Y.
  const int32_t* gather_rows;
  int gather_src_rows;
  int k_red2;            // kModeRows: > 0 adds a second contraction segment into the same
                         // accumulator: C = A . op(B[g]) + A2 . op(B2[g]), A2 [m_total,
                         // k_red2] through map_c2 and B2 through map_b2 (two-segment dgrad)
};

struct TileInfo {
  int g;       // expert
  int m_blk;   // tile row block (TILE_M rows)
  int n_blk;   // tile column block (BN columns)
  int row0;    // kModeRows: first A row of the tile; kModeWgrad: first row of the expert
  int rows;    // kModeRows: valid output rows of the tile; kModeWgrad: rows of the expert
  int nkb;     // number of 64-deep contraction blocks
};

// First row and row count of expert g (negative counts clamp to zero).
__device__ __forceinline__ void group_range(const Params& p, int g, int& start, int& rows) {
  int st, en;
  if (p.offsets_plus_one) { st = __ldg(p.offsets + g); en = __ldg(p.offsets + g + 1); }
  else { st = g > 0 ? __ldg(p.offsets + g - 1) : 0; en = __ldg(p.offsets + g); }
  start = st;
  rows = en > st ? en - st : 0;
}

template <int MODE, int CG>
__device__ __forceinline__ int tiles_of_group(const Params& p, int rows) {
  constexpr int TM = Shape<CG>::TILE_M;
  const int nt = (p.n_out + tile_out_cols<MODE>() - 1) / tile_out_cols<MODE>();
  if (MODE != kModeWgrad) return ((rows + TM - 1) / TM) * nt;
  return ((p.p_out + TM - 1) / TM) * nt;
}

template <int MODE, int CG>
__device__ __forceinline__ TileInfo decode_tile(const int* tile_prefix, const Params& p, int t) {
  constexpr int TM = Shape<CG>::TILE_M;
  // Largest g with tile_prefix[g] <= t; experts that own no tile are skipped because
  // their prefix equals the next expert's.
  int lo = 0, hi = p.num_groups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tile_prefix[mid] <= t) lo = mid; else hi = mid - 1;
  }
  TileInfo ti;
  ti.g = lo;
  const int local = t - tile_prefix[lo];
  int start, rows;
  group_range(p, lo, start, rows);
  if (MODE != kModeWgrad) {
    const int mt = (rows + TM - 1) / TM;
    ti.m_blk = local % mt;
    ti.n_blk = local / mt;
    ti.row0 = start + ti.m_blk * TM;
    ti.rows = min(TM, rows - ti.m_blk * TM);
    ti.nkb = (p.k_red + BK - 1) / BK + (p.k_red2 + BK - 1) / BK;
  } else {
    if (p.q_fastest) {
      // Concurrent tiles cover whole output rows: each row of the gradient is written in
      // one burst of adjacent column blocks instead of one block at a time.
      const int nt = (p.n_out + BN - 1) / BN;
      ti.n_blk = local % nt;
      ti.m_blk = local / nt;
    } else {
      const int pt = (p.p_out + TM - 1) / TM;
      ti.m_blk = local % pt;
      ti.n_blk = local / pt;
    }
    ti.row0 = start;
    ti.rows = rows;
    ti.nkb = (rows + BK - 1) / BK;
  }
  return ti;
}

// A half tile is the last row tile of an expert in an SM pair when it holds at most 128
// rows: the pair then runs cta_group::2 MMAs with M = 128, each CTA holding 64 rows of A
// (and of the accumulator), so a short tail costs half a pair tile instead of a full one.
// The accumulator of such a tile sits in TMEM as 64 rows x 256 columns per CTA folded into
// 128 lanes x 128 columns: lanes 0-63 hold columns 0-127 and lanes 64-127 hold columns
// 128-255 of rows 0-63.
template <int MODE, int CG>
__device__ __forceinline__ bool is_half_tile(const TileInfo& ti) {
  return MODE == kModeRows && CG == 2 && ti.rows <= BMC;
}

// Packs 8 fp32 values into 8 16-bit values (round to nearest even) as one 16-byte vector.
template <typename OutT>
__device__ __forceinline__ uint4 pack8_16b(const uint32_t* v) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = __uint_as_float(v[2 * i]), hi = __uint_as_float(v[2 * i + 1]);
    if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
      __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(lo, hi);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Pipeline waits are CTA-scope acquires: data hand-offs between the two CTAs of a pair
// are ordered by TMA transaction counts and tcgen05 commits, not by generic memory.
__device__ __forceinline__ bool wait_local(uint32_t bar, uint32_t parity, volatile int* abort) {
  return ptx::wait_bounded(bar, parity, abort, kWaitTimeoutNs);
}

// Stores one 32 x 32 block of 16-bit values held row per lane (`wd`: this lane's row,
// 16 words) through the warp's 2 KB staging buffer: with a TMA store at (x, y) of `map` when
// the block's 32 rows are all valid (the store clips columns at the tensor's edge), else
// with 16-byte stores of the valid rows and columns at dst (element (0, 0) of the block,
// row pitch `ld` elements).
template <typename OutT>
__device__ __forceinline__ void stage_store_block(const uint32_t* wd, uint8_t* cbuf, uint32_t cbuf_u32,
                                                  int lane, bool use_tma, const CUtensorMap* map,
                                                  int x, int y, OutT* dst, int64_t ld,
                                                  int valid_rows, int valid_cols) {
  if (lane == 0) ptx::bulk_wait_group_read<0>();  // the previous store has read the buffer
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int phys = i ^ ((lane >> 1) & 3);
    *reinterpret_cast<uint4*>(cbuf + lane * 64 + phys * 16) =
        make_uint4(wd[i * 4 + 0], wd[i * 4 + 1], wd[i * 4 + 2], wd[i * 4 + 3]);
  }
  if (use_tma) {
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      ptx::tma_store_2d(map, cbuf_u32, x, y);
      ptx::bulk_commit_group();
    }
    return;
  }
  __syncwarp();
  const int chunk = lane & 3, cc = chunk * 8;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rr = (lane >> 2) + i * 8;
    const int phys = chunk ^ ((rr >> 1) & 3);
    const uint4 u = *reinterpret_cast<const uint4*>(cbuf + rr * 64 + phys * 16);
    if (rr < valid_rows && cc < valid_cols) *reinterpret_cast<uint4*>(dst + (int64_t)rr * ld + cc) = u;
  }
  __syncwarp();
}

// Packs 32 fp32 values (as bits) into 16 words of 16-bit values.
template <typename OutT>
__device__ __forceinline__ void pack32_16b(const uint32_t* v, uint32_t* wd) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 x = pack8_16b<OutT>(&v[i * 8]);
    wd[i * 4 + 0] = x.x; wd[i * 4 + 1] = x.y; wd[i * 4 + 2] = x.z; wd[i * 4 + 3] = x.w;
  }
}

// A_MN / B_MN: the operand is MN-major in global memory (and in shared memory).
// In kModeRows map_b is 3-D (inner, outer, expert); every other map is 2-D (inner, row).
// Tensor-map boxes: A 64 x 128 (K-major) or 64 x 64 (MN-major, 2 per CTA); B 64 x B_COLS
// (K-major) or 64 x 64 (MN-major, B_COLS / 64 per CTA).
template <int MODE, int CG, int AB_FORMAT, bool A_MN, bool B_MN, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
gmm_sm100_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                 const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_b2,
                 const __grid_constant__ CUtensorMap map_c2, const __grid_constant__ CUtensorMap map_c3,
                 const Params p) {
  static_assert((MODE != kModeGateUp && MODE != kModeSwiGLUBwd) || CG == 1,
                "fused-epilogue tiles run on single CTAs");
  using Sh = Shape<CG>;
  constexpr int STAGES = Sh::STAGES;
  extern __shared__ uint8_t smem_raw[];
  SmemLayout<CG>& s = *reinterpret_cast<SmemLayout<CG>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &s.abort;
  const uint32_t rank = CG == 1 ? 0u : ptx::cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster_id = blockIdx.x / CG;
  const int num_clusters = gridDim.x / CG;

  // ------------------------------------------------------------ prologue
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      ptx::mbar_init(ptx::smem_u32(&s.full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&s.empty[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&s.peer_done[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&s.raw[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(ptx::smem_u32(&s.tmem_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&s.tmem_empty[i]), CG * kEpiWarps);
    }
    s.abort = 0;
    ptx::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&map_a);
    ptx::prefetch_tensormap(&map_b);
    ptx::prefetch_tensormap(&map_c);
    if (MODE == kModeGateUp) {
      ptx::prefetch_tensormap(&map_b2);
      ptx::prefetch_tensormap(&map_c2);
      ptx::prefetch_tensormap(&map_c3);
    }
    if (MODE == kModeRows && p.k_red2 > 0) {
      ptx::prefetch_tensormap(&map_b2);
      ptx::prefetch_tensormap(&map_c2);
    }
  }
  if (warp == 1) {
    ptx::tmem_alloc<CG>(ptx::smem_u32(&s.tmem_base), kTmemCols);
    ptx::tmem_relinquish<CG>();
  }
  // Per-expert tile prefix (block-wide scan; each thread owns up to PER experts).
  {
    constexpr int PER = (kMaxGroups + kThreads - 1) / kThreads;
    const int g0 = threadIdx.x * PER;
    int cnt[PER];
    int local_sum = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int g = g0 + i;
      cnt[i] = 0;
      if (g < p.num_groups) {
        int st, rows;
        group_range(p, g, st, rows);
        cnt[i] = tiles_of_group<MODE, CG>(p, rows);
      }
      local_sum += cnt[i];
    }
    int incl = local_sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    if (lane == 31) s.warp_sums[warp] = incl;
    __syncthreads();
    int warp_base = 0;
    for (int w = 0; w < warp; ++w) warp_base += s.warp_sums[w];
    int run = warp_base + incl - local_sum;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int g = g0 + i;
      if (g < p.num_groups) s.tile_prefix[g] = run;
      run += cnt[i];
    }
    if (threadIdx.x == kThreads - 1) s.tile_prefix[p.num_groups] = run;
  }
  ptx::tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) ptx::cluster_sync();  // peer barriers are initialised
  ptx::tc_fence_after();
  const int total_tiles = s.tile_prefix[p.num_groups];
  const uint32_t tmem_base = s.tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    // Never waits on data: a masked wgrad block is loaded on the stage's `raw` barrier and
    // handed to the fix-up warp, the producer moves on to the next stage.
    int stage = 0;
    uint32_t phase = 0;
    const bool gather = p.gather_rows != nullptr;
    // A source row of the gathered operand, clamped into the tensor (rows past the data
    // are never stored: row tiles mask them and wgrad zeroes them).
    auto src_row = [&](int r) {
      r = min(max(r, 0), (int)p.m_total - 1);
      const int v = __ldg(p.gather_rows + r);
      return min(max(v, 0), p.gather_src_rows - 1);
    };
    for (int t = cluster_id; t < total_tiles && !*abort_flag; t += num_clusters) {
      const TileInfo ti = decode_tile<MODE, CG>(s.tile_prefix, p, t);
      int grow[4] = {0, 0, 0, 0};  // row tiles: this lane's 4 rows of the tile's A block
      if (MODE != kModeWgrad && gather) {
#pragma unroll
        for (int i = 0; i < 4; ++i) grow[i] = src_row(ti.row0 + lane * 4 + i);
      }
      for (int kb = 0; kb < ti.nkb; ++kb) {
        if (!wait_local(ptx::smem_u32(&s.empty[stage]), phase ^ 1, abort_flag)) break;
        if (MODE == kModeWgrad && gather) {
          // this lane's 4 contraction rows of the k-block (16 groups of 4 per 64 rows)
          const int r = ti.row0 + kb * BK + (lane & 15) * 4;
#pragma unroll
          for (int i = 0; i < 4; ++i) grow[i] = src_row(r + i);
        }
        if (lane == 0) {
          const uint32_t sa = ptx::smem_u32(&s.a[stage][0]);
          const uint32_t sb = ptx::smem_u32(&s.b[stage][0]);
          // The leader's full barrier, addressed for the cluster.
          const uint32_t full_local = ptx::smem_u32(&s.full[stage]);
          const uint32_t full_c = CG == 1 ? full_local : ptx::mapa_shared(full_local, 0);
          if (MODE != kModeWgrad) {
            // The leader expects the bytes of both CTAs; the peer's loads complete their
            // bytes on the leader's barrier (possibly before this expect, which is fine:
            // the phase cannot complete before the leader's single arrival).  A comes in
            // 64-row boxes: two per CTA, or one for a half tile.
            const bool half = is_half_tile<MODE, CG>(ti);
            if (leader)
              ptx::mbar_arrive_expect_tx(
                  full_local, CG * (half ? Sh::STAGE_BYTES - Sh::A_BYTES / 2 : Sh::STAGE_BYTES));
            // Two-segment row tiles: the k-blocks past the first segment's come from the
            // second operand pair (A2 through map_c2, B2 through map_b2).
            const int nkb1 = (p.k_red + BK - 1) / BK;
            const bool seg2 = MODE == kModeRows && kb >= nkb1;
            const int k0 = (seg2 ? kb - nkb1 : kb) * BK;
            const CUtensorMap* mapA = seg2 ? &map_c2 : &map_a;
            const CUtensorMap* mapB = seg2 ? &map_b2 : &map_b;
            const int nb = ti.n_blk * tile_out_cols<MODE>() + (int)rank * Sh::B_COLS;
            const int a_rows = half ? BMC / 2 : BMC;
            for (int j = 0; j < a_rows / 64 && !gather; ++j) {
              const int ar = ti.row0 + (int)rank * a_rows + j * 64;
              if (CG == 1) ptx::tma_load_2d(sa + j * (64 * 128), mapA, full_c, k0, ar);
              else ptx::tma_load_2d_pair(sa + j * (64 * 128), mapA, full_c, k0, ar);
            }
            if (MODE == kModeGateUp) {
              // B rows 0-127: gate columns nb.., rows 128-255: the same up columns.
              if (!B_MN) {
                ptx::tma_load_3d(sb, &map_b, full_c, k0, nb, ti.g);
                ptx::tma_load_3d(sb + (BN / 2) * 128, &map_b2, full_c, k0, nb, ti.g);
              } else {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                  ptx::tma_load_3d(sb + j * (BK * 128), &map_b, full_c, nb + j * 64, k0, ti.g);
                  ptx::tma_load_3d(sb + (2 + j) * (BK * 128), &map_b2, full_c, nb + j * 64, k0, ti.g);
                }
              }
            } else if (!B_MN) {
              if (CG == 1) ptx::tma_load_3d(sb, mapB, full_c, k0, nb, ti.g);
              else ptx::tma_load_3d_pair(sb, mapB, full_c, k0, nb, ti.g);
            } else {
#pragma unroll
              for (int j = 0; j < Sh::B_COLS / 64; ++j) {
                if (CG == 1) ptx::tma_load_3d(sb + j * (BK * 128), mapB, full_c, nb + j * 64, k0, ti.g);
                else ptx::tma_load_3d_pair(sb + j * (BK * 128), mapB, full_c, nb + j * 64, k0, ti.g);
              }
            }
          } else {
            const int r0 = ti.row0 + kb * BK;
            const bool masked = ti.row0 + ti.rows - r0 < BK;  // block reaches past the expert
            const int pa = ti.m_blk * Sh::TILE_M + (int)rank * BMC;
            const int qb = ti.n_blk * BN + (int)rank * Sh::B_COLS;
            if (!masked) {
              if (leader) ptx::mbar_arrive_expect_tx(full_local, CG * Sh::STAGE_BYTES);
#pragma unroll
              for (int j = 0; j < BMC / 64; ++j) {
                if (CG == 1) ptx::tma_load_2d(sa + j * (BK * 128), &map_a, full_c, pa + j * 64, r0);
                else ptx::tma_load_2d_pair(sa + j * (BK * 128), &map_a, full_c, pa + j * 64, r0);
              }
#pragma unroll
              for (int j = 0; j < Sh::B_COLS / 64; ++j) {
                if (gather) break;
                if (CG == 1) ptx::tma_load_2d(sb + j * (BK * 128), &map_b, full_c, qb + j * 64, r0);
                else ptx::tma_load_2d_pair(sb + j * (BK * 128), &map_b, full_c, qb + j * 64, r0);
              }
            } else {
              const uint32_t rb = ptx::smem_u32(&s.raw[stage]);
              ptx::mbar_arrive_expect_tx(rb, Sh::STAGE_BYTES);
#pragma unroll
              for (int j = 0; j < BMC / 64; ++j)
                ptx::tma_load_2d(sa + j * (BK * 128), &map_a, rb, pa + j * 64, r0);
#pragma unroll
              for (int j = 0; j < Sh::B_COLS / 64; ++j) {
                if (gather) break;
                ptx::tma_load_2d(sb + j * (BK * 128), &map_b, rb, qb + j * 64, r0);
              }
            }
          }
        }
        if (gather) {
          // The gathered operand: every lane fetches 4 rows with one gather4 per 64-column
          // box (its bytes are in the stage's expect_tx armed by lane 0 above).
          __syncwarp();
          const uint32_t sa = ptx::smem_u32(&s.a[stage][0]);
          const uint32_t sb = ptx::smem_u32(&s.b[stage][0]);
          const uint32_t full_local = ptx::smem_u32(&s.full[stage]);
          const uint32_t full_c = CG == 1 ? full_local : ptx::mapa_shared(full_local, 0);
          if (MODE != kModeWgrad) {
            ptx::tma_gather4(sa + lane * 512, &map_a, full_c, kb * BK, grow[0], grow[1], grow[2],
                             grow[3]);
          } else {
            const int r0 = ti.row0 + kb * BK;
            const bool masked = ti.row0 + ti.rows - r0 < BK;
            const int qb = ti.n_blk * BN + (int)rank * Sh::B_COLS;
            const uint32_t bar = masked ? ptx::smem_u32(&s.raw[stage]) : full_c;
            for (int j = lane >> 4; j < Sh::B_COLS / 64; j += 2) {
              const uint32_t dst = sb + j * (BK * 128) + (lane & 15) * 512;
              if (CG == 1 || masked)
                ptx::tma_gather4(dst, &map_b, bar, qb + j * 64, grow[0], grow[1], grow[2], grow[3]);
              else
                ptx::tma_gather4_pair(dst, &map_b, bar, qb + j * 64, grow[0], grow[1], grow[2],
                                      grow[3]);
            }
          }
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else if (MODE == kModeWgrad && warp == 2) {
    // ---------------------------------------------------------- masked-block fix-up
    // Walks the same stage sequence as the producer.  For a block that reaches past the
    // expert's last row: wait for its data on `raw`, zero the rows past the expert (a
    // swizzled 128-byte row stays one row), fence the generic->async proxy, then hand the
    // stage to the MMA (for a pair, the peer releases its rows to the leader first).
    int stage = 0;
    uint32_t raw_bits = 0, peer_bits = 0;  // per-stage parities
    for (int t = cluster_id; t < total_tiles && !*abort_flag; t += num_clusters) {
      const TileInfo ti = decode_tile<MODE, CG>(s.tile_prefix, p, t);
      bool ok = true;
      for (int kb = 0; kb < ti.nkb && ok; ++kb) {
        const int r0 = ti.row0 + kb * BK;
        const int valid = ti.row0 + ti.rows - r0;
        if (valid < BK) {
          const uint32_t rb = ptx::smem_u32(&s.raw[stage]);
          ok = ptx::wait_bounded(rb, (raw_bits >> stage) & 1u, abort_flag, kWaitTimeoutNs);
          raw_bits ^= 1u << stage;
          if (!ok) break;
          const int n16 = (BK - valid) * 8;  // 16-byte chunks to clear per 64-column box
          constexpr int kBoxes = (BMC + Sh::B_COLS) / 64;
          for (int box = 0; box < kBoxes; ++box) {
            uint8_t* base = box < BMC / 64 ? &s.a[stage][box * BK * 128]
                                           : &s.b[stage][(box - BMC / 64) * BK * 128];
            for (int i = lane; i < n16; i += 32)
              reinterpret_cast<uint4*>(base + valid * 128)[i] = make_uint4(0, 0, 0, 0);
          }
          ptx::fence_proxy_async_smem();
          __syncwarp();
          const uint32_t full_local = ptx::smem_u32(&s.full[stage]);
          if (CG == 1) {
            if (lane == 0) ptx::mbar_arrive(full_local);
          } else if (!leader) {
            if (lane == 0)
              ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_u32(&s.peer_done[stage]), 0));
          } else {
            const uint32_t pd = ptx::smem_u32(&s.peer_done[stage]);
            ok = ptx::wait_bounded_cluster(pd, (peer_bits >> stage) & 1u, abort_flag,
                                           kWaitTimeoutNs);
            peer_bits ^= 1u << stage;
            if (!ok) break;
            if (lane == 0) ptx::mbar_arrive(full_local);
          }
          __syncwarp();
        }
        if (++stage == STAGES) stage = 0;
      }
      if (!ok) break;
    }
  } else if (warp == 1 && leader) {
    // ---------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc =
        ptx::make_idesc_f16(AB_FORMAT, A_MN ? 1 : 0, B_MN ? 1 : 0, Sh::TILE_M, BN);
    constexpr uint32_t idesc_half =
        ptx::make_idesc_f16(AB_FORMAT, A_MN ? 1 : 0, B_MN ? 1 : 0, BMC, BN);
    // K-major: rows of 128 bytes, 8-row atoms 1024 bytes apart; a K=16 step is +32 bytes.
    // MN-major: 64-element column chunks BK*128 bytes apart (LBO), 8-k-row atoms 1024
    // bytes apart (SBO); a K=16 step is two atoms (+2048 bytes).
    constexpr uint32_t kLboMN = BK * 128;
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    for (int t = cluster_id; t < total_tiles && !*abort_flag; t += num_clusters, ++acc) {
      const TileInfo ti = decode_tile<MODE, CG>(s.tile_prefix, p, t);
      const int buf = acc & 1;
      const uint32_t acc_phase = (acc >> 1) & 1;
      if (!wait_local(ptx::smem_u32(&s.tmem_empty[buf]), acc_phase ^ 1, abort_flag)) break;
      ptx::tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * BN;
      const uint32_t tile_idesc = is_half_tile<MODE, CG>(ti) ? idesc_half : idesc;
      bool ok = true;
      for (int kb = 0; kb < ti.nkb; ++kb) {
        if (!wait_local(ptx::smem_u32(&s.full[stage]), phase, abort_flag)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        if (lane == 0) {
          const uint32_t sa = ptx::smem_u32(&s.a[stage][0]);
          const uint32_t sb = ptx::smem_u32(&s.b[stage][0]);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint64_t ad = A_MN ? ptx::make_sw128_desc(sa + kk * 2048, kLboMN, 1024)
                                     : ptx::make_sw128_desc(sa + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? ptx::make_sw128_desc(sb + kk * 2048, kLboMN, 1024)
                                     : ptx::make_sw128_desc(sb + kk * 32, 16, 1024);
            ptx::mma_f16_ss<CG>(d_tmem, ad, bd, tile_idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          const uint32_t eb = ptx::smem_u32(&s.empty[stage]);
          ptx::mma_commit<CG>(eb);
          if (CG == 2) ptx::mma_commit<CG>(ptx::mapa_shared(eb, 1));
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (lane == 0) {
        const uint32_t fb = ptx::smem_u32(&s.tmem_full[buf]);
        if (ti.nkb > 0) {
          ptx::mma_commit<CG>(fb);
          if (CG == 2) ptx::mma_commit<CG>(ptx::mapa_shared(fb, 1));
        } else {
          ptx::mbar_arrive(fb);
          if (CG == 2) ptx::mbar_arrive_relaxed_cluster(ptx::mapa_shared(fb, 1));
        }
      }
      __syncwarp();
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------- epilogue
    // Warp w reads TMEM lanes 32*(w%4)..+31 (this CTA's tile rows) and columns
    // [128*h, 128*h+128), h = (w-4)/4, in four 32-column chunks.  Each chunk is rounded to
    // 16 bits, written row-per-lane into a 2 KB buffer (16-byte chunks XOR-swizzled so both
    // the row-wise writes and the column-wise reads are conflict-free), read back so that
    // every store instruction writes eight full 64-byte row segments, and stored with a
    // row/column mask.  The next chunk's TMEM load is issued before the current chunk is
    // stored.
    const int ew = warp - 4;
    const int q = ew & 3, h = ew >> 2;
    OutT* out = static_cast<OutT*>(p.out);
    uint8_t* cbuf = &s.cbuf[ew][0][0];
    const int wr_row = lane;        // row written by this lane
    const int rd_chunk = lane & 3;  // 16-byte chunk read by this lane
    const int rd_row0 = lane >> 2;  // first row read by this lane (then +8, +16, +24)
    const uint32_t cbuf_u32 = ptx::smem_u32(cbuf);
    constexpr int kBufs = Sh::EPI_BUFS;
    int chunk_ctr = 0;  // 32 x 32 blocks this warp has staged (selects the buffer)
    int acc = 0;
    for (int t = cluster_id; t < total_tiles && !*abort_flag; t += num_clusters, ++acc) {
      const TileInfo ti = decode_tile<MODE, CG>(s.tile_prefix, p, t);
      const int buf = acc & 1;
      const uint32_t acc_phase = (acc >> 1) & 1;
      if constexpr (MODE == kModeSwiGLUBwd) {
        // While this tile's main loop runs, pull the gate / up values its epilogue will
        // read into L2: this lane's row, the warp's 128 columns (256 bytes, up to 3 lines).
        const int r = q * 32 + lane;
        const int c0 = ti.n_blk * BN + h * (BN / 2);
        if (r < min(BMC, ti.rows) && c0 < p.n_out) {
          const int64_t e0 = (int64_t)(ti.row0 + r) * p.n_out + c0;
          const int64_t e1 = e0 + min(BN / 2, p.n_out - c0) - 1;  // last element
          const OutT* gsrc = static_cast<const OutT*>(p.in_gate);
          const OutT* usrc = static_cast<const OutT*>(p.in_up);
          for (int64_t e = e0; e <= e1 + 63; e += 64) {
            const int64_t ee = e < e1 ? e : e1;
            ptx::prefetch_l2(gsrc + ee);
            ptx::prefetch_l2(usrc + ee);
          }
        }
      }
      if (!wait_local(ptx::smem_u32(&s.tmem_full[buf]), acc_phase, abort_flag)) break;
      ptx::tc_fence_after();
      if constexpr (MODE == kModeGateUp) {
        // Warp (q, h) owns rows 32q..32q+31 and output columns [64h, 64h+64) of the tile:
        // two 32-column chunks, each read from the gate half (TMEM column c) and the up half
        // (column 128 + c) of the accumulator.  gate and up are rounded to 16 bits as the
        // plain GEMM stores them, then h = rnd(rnd(silu(gate)) * up) as the SwiGLU kernel
        // computes it, so the three outputs equal GEMM + GEMM + SwiGLU bit for bit.
        const int n0 = ti.n_blk * (BN / 2);
        const int valid_cols = min(BN / 2, p.n_out - n0);
        const int valid_rows = min(BMC, ti.rows);
        const int row_base = ti.row0;
        const bool use_tma = (q + 1) * 32 <= valid_rows;
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
        const int vr = min(32, valid_rows - q * 32);
        OutT* const outs[3] = {static_cast<OutT*>(p.out_gate), static_cast<OutT*>(p.out_up), out};
        const CUtensorMap* const maps[3] = {&map_c2, &map_c3, &map_c};
        if (vr > 0) {
          for (int c = 0; c < 2; ++c) {
            const int col = h * 64 + c * 32;
            if (col >= valid_cols) break;
            uint32_t vg[32], vu[32], wd[16];
            ptx::tmem_ld_32x32b_x32(tbase + col, vg);
            ptx::tmem_ld_32x32b_x32(tbase + BN / 2 + col, vu);
            ptx::tmem_wait_ld();
            const int64_t off = (int64_t)(row_base + q * 32) * p.n_out + n0 + col;
#pragma unroll
            for (int o = 0; o < 3; ++o) {
              if (o == 0) pack32_16b<OutT>(vg, wd);
              else if (o == 1) pack32_16b<OutT>(vu, wd);
              else {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                  const float gq = rnd<OutT>(__uint_as_float(vg[i]));
                  const float uq = rnd<OutT>(__uint_as_float(vu[i]));
                  vg[i] = __float_as_uint(rnd<OutT>(gq * sigmoid_f32(gq)) * uq);
                }
                pack32_16b<OutT>(vg, wd);
              }
              stage_store_block<OutT>(wd, cbuf, cbuf_u32, lane, use_tma, maps[o], n0 + col,
                                      row_base + q * 32, outs[o] + off, p.n_out, vr,
                                      valid_cols - col);
            }
          }
        }
      } else if constexpr (MODE == kModeSwiGLUBwd) {
        // The tile's accumulator is the gradient of h (rows 32q.., columns [128h, 128h+128)
        // for this warp, four 32-column chunks).  Each lane loads its row's gate and up values,
        // rounds the gradient to 16 bits as the plain GEMM stores it, and applies the SwiGLU
        // backward exactly as the SwiGLU backward kernel does, so grad_gate and grad_up equal
        // dgrad GEMM + SwiGLU backward bit for bit.
        const int n0 = ti.n_blk * BN;
        const int valid_cols = min(BN, p.n_out - n0);
        const int valid_rows = min(BMC, ti.rows);
        const int row_base = ti.row0;
        const bool use_tma = (q + 1) * 32 <= valid_rows;
        const int vr = min(32, valid_rows - q * 32);
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
        const OutT* gin = static_cast<const OutT*>(p.in_gate);
        const OutT* uin = static_cast<const OutT*>(p.in_up);
        OutT* dg_out = out;
        OutT* du_out = static_cast<OutT*>(p.out_up);
        const bool row_ok = q * 32 + lane < valid_rows;
        const int64_t my_row = (int64_t)(row_base + q * 32 + lane) * p.n_out;
        if (vr > 0) {
          for (int c = 0; c < 4; ++c) {
            const int col = h * (BN / 2) + c * 32;
            if (col >= valid_cols) break;
            uint32_t v[32];
            ptx::tmem_ld_32x32b_x32(tbase + col, v);
            uint4 graw[4], uraw[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const bool ok = row_ok && col + i * 8 < valid_cols;
              graw[i] = ok ? __ldg(reinterpret_cast<const uint4*>(gin + my_row + n0 + col + i * 8))
                           : make_uint4(0, 0, 0, 0);
              uraw[i] = ok ? __ldg(reinterpret_cast<const uint4*>(uin + my_row + n0 + col + i * 8))
                           : make_uint4(0, 0, 0, 0);
            }
            ptx::tmem_wait_ld();
            const OutT* gv = reinterpret_cast<const OutT*>(graw);
            const OutT* uv = reinterpret_cast<const OutT*>(uraw);
            uint32_t vdg[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              float a, b;
              swiglu_bwd_elem<OutT>(rnd<OutT>(__uint_as_float(v[i])), to_f32(gv[i]), to_f32(uv[i]),
                                    a, b);
              vdg[i] = __float_as_uint(a);
              v[i] = __float_as_uint(b);
            }
            uint32_t wd[16];
            const int64_t off = (int64_t)(row_base + q * 32) * p.n_out + n0 + col;
            pack32_16b<OutT>(vdg, wd);
            stage_store_block<OutT>(wd, cbuf, cbuf_u32, lane, use_tma, &map_c, n0 + col,
                                    row_base + q * 32, dg_out + off, p.n_out, vr, valid_cols - col);
            pack32_16b<OutT>(v, wd);
            stage_store_block<OutT>(wd, cbuf, cbuf_u32, lane, use_tma, &map_c3, n0 + col,
                                    row_base + q * 32, du_out + off, p.n_out, vr, valid_cols - col);
          }
        }
      } else {
        const int n0 = ti.n_blk * BN;
        // Full tile: this warp reads TMEM lanes of rows 32q..32q+31 and tile columns
        // [128h, 128h+128).  Half tile: lanes 32q.. hold rows 32(q&1).. of the CTA's 64 and
        // tile columns from 128(q>>1); the warp reads 64 of those columns from TMEM column 64h.
        const bool half = is_half_tile<MODE, CG>(ti);
        const int rq = half ? (q & 1) : q;                 // 32-row group of this warp
        const int tcol = half ? h * 64 : h * (BN / 2);    // first TMEM column read
        const int col_lo = half ? (q >> 1) * (BN / 2) + h * 64 : h * (BN / 2);
        const int ncols = half ? 64 : BN / 2;
        const int valid_cols = min(BN, p.n_out - n0);
        int valid_rows, row_base;
        OutT* tile_ptr;  // element (0, 0) of this CTA's rows of the tile
        if (MODE == kModeRows) {
          const int cta_rows = half ? BMC / 2 : BMC;
          valid_rows = min(cta_rows, ti.rows - (int)rank * cta_rows);
          row_base = ti.row0 + (int)rank * cta_rows;
          tile_ptr = out + (int64_t)row_base * p.n_out + n0;
        } else {
          row_base = ti.m_blk * Sh::TILE_M + (int)rank * BMC;  // row inside expert g
          valid_rows = min(BMC, p.p_out - row_base);
          tile_ptr = out + ((int64_t)ti.g * p.p_out + row_base) * p.n_out + n0;
        }
        // TMA stores clip at the output's edges, so they serve every wgrad tile and every
        // warp whose 32 rows all belong to the expert; the others store with masks so they
        // never touch the next expert's rows.  A warp with no valid row stores nothing.
        const bool use_tma = MODE == kModeWgrad || (rq + 1) * 32 <= valid_rows;
        const int nchunks = (MODE == kModeRows && valid_rows <= rq * 32)
                                ? 0
                                : max(0, min(ncols, valid_cols - col_lo) + 31) / 32;
        const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN + tcol;
        uint32_t v[32];
        const bool has_acc = ti.nkb > 0;
        if (has_acc && nchunks > 0) {
          ptx::tmem_ld_32x32b_x32(tbase, v);
          ptx::tmem_wait_ld();
        }
        for (int c = 0; c < nchunks; ++c) {
          uint32_t w[16];
          if (has_acc) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint4 u = pack8_16b<OutT>(&v[i * 8]);
              w[i * 4 + 0] = u.x; w[i * 4 + 1] = u.y; w[i * 4 + 2] = u.z; w[i * 4 + 3] = u.w;
            }
            if (c + 1 < nchunks) ptx::tmem_ld_32x32b_x32(tbase + (c + 1) * 32, v);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) w[i] = 0u;
          }
          // The TMA store that last used this buffer must have finished reading it: with
          // kBufs buffers in rotation, at most kBufs - 1 later stores may still be reading.
          // The masked path below reads its buffer back without a store group, so it waits
          // for all of them.
          uint8_t* cb = cbuf + (chunk_ctr % kBufs) * kEpiBufBytes;
          const uint32_t cb_u32 = cbuf_u32 + (uint32_t)((chunk_ctr % kBufs) * kEpiBufBytes);
          ++chunk_ctr;
          if (lane == 0) {
            if (use_tma) ptx::bulk_wait_group_read<kBufs - 1>();
            else ptx::bulk_wait_group_read<0>();
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int phys = i ^ ((wr_row >> 1) & 3);
            *reinterpret_cast<uint4*>(cb + wr_row * 64 + phys * 16) =
                make_uint4(w[i * 4 + 0], w[i * 4 + 1], w[i * 4 + 2], w[i * 4 + 3]);
          }
          if (use_tma) {
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              const int cx = n0 + col_lo + c * 32;
              if (MODE == kModeRows) ptx::tma_store_2d(&map_c, cb_u32, cx, row_base + rq * 32);
              else ptx::tma_store_3d(&map_c, cb_u32, cx, row_base + rq * 32, ti.g);
              ptx::bulk_commit_group();
            }
            if (has_acc && c + 1 < nchunks) ptx::tmem_wait_ld();
            continue;
          }
          __syncwarp();
          const int col = col_lo + c * 32 + rd_chunk * 8;  // first column of this lane's chunk
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = rd_row0 + i * 8;
            const int phys = rd_chunk ^ ((rr >> 1) & 3);
            const uint4 u = *reinterpret_cast<const uint4*>(cb + rr * 64 + phys * 16);
            const int row = rq * 32 + rr;
            if (row < valid_rows && col < valid_cols)
              *reinterpret_cast<uint4*>(tile_ptr + (int64_t)row * p.n_out + col) = u;
          }
          __syncwarp();
          if (has_acc && c + 1 < nchunks) ptx::tmem_wait_ld();
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        // TMEM reads are complete (tcgen05.wait::ld); the stores need no ordering here.
        const uint32_t eb = ptx::smem_u32(&s.tmem_empty[buf]);
        if (leader) ptx::mbar_arrive(eb);
        else ptx::mbar_arrive_relaxed_cluster(ptx::mapa_shared(eb, 0));
      }
    }
    // The TMA stores must have landed before the CTA ends.
    if (lane == 0) ptx::bulk_wait_group<0>();
    __syncwarp();
  }

  // ------------------------------------------------------------ teardown
  __syncthreads();
  if (*abort_flag) {
    if (threadIdx.x == 0) raise_device_error(1);
    // Let any copy or MMA that was still in flight land before the memory is released.
    if (warp == 1) __nanosleep(100000);
    __syncwarp();
  }
  if constexpr (CG == 2) ptx::cluster_sync();  // no remote arrivals target this CTA any more
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc<CG>(tmem_base, kTmemCols);
  }
}

}  // namespace gmm
}  // namespace moe
