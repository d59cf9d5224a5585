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
// Warp roles (256 threads, one CTA per SM, persistent over a static tile stride):
//   warp 0     TMA producer: fills a 4-stage shared-memory ring (A 128x64, B 256x64 per
//              stage, 128-byte swizzle) and signals `full[s]` with the transaction bytes.
//   warp 1     TMEM owner and MMA issuer: one elected thread issues 4 tcgen05.mma
//              (M=128, N=256, K=16) per stage into one of two TMEM accumulators
//              (2 x 256 fp32 columns) and commits each stage back to `empty[s]`.
//   warps 4-7  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//              32*(w%4)..+31, i.e. output rows), round to the output dtype and store with
//              16-byte vector stores, masking rows past the expert's end and columns past
//              the output width.  Releasing the accumulator lets the MMA warp start the
//              tile after next, so the epilogue overlaps the next tile's main loop.
//
// Ragged contraction (wgrad): the last 64-row block of an expert may reach into the next
// expert's rows.  The producer loads that block on a private barrier, zeroes the rows
// past the expert's end in shared memory (a swizzled 128-byte row stays one row), fences
// the generic->async proxy and then arrives on `full[s]` itself.
//
// Tile scheduler: each CTA builds the per-expert tile prefix from `offsets` in shared
// memory (no host sync), then walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...  Inside
// an expert, tiles run row-block fastest so that the CTAs working at the same time share
// the same B tile through L2.  Empty experts own no tile in kModeRows; in kModeWgrad they
// own their full [P, Q] tiles, written as zeros.
//
// Every mbarrier wait is bounded (2 s); a wait that gives up sets a shared abort flag and
// the device error word, every role then leaves its loop and the TMEM is freed.
#pragma once

#include "common.cuh"
#include "sm100_ptx.cuh"

#include <type_traits>

namespace moe {
namespace gmm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;  // 64 x 16-bit = one 128-byte swizzle row
constexpr int STAGES = 4;
constexpr int UMMA_K = 16;
constexpr int kThreads = 256;
constexpr int kMaxGroups = 1024;
constexpr uint32_t A_STAGE_BYTES = BM * BK * 2;
constexpr uint32_t B_STAGE_BYTES = BN * BK * 2;
constexpr uint32_t STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr uint32_t kTmemCols = 2 * BN;
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

enum Mode { kModeRows = 0, kModeWgrad = 1 };

struct SmemLayout {
  uint8_t a[STAGES][A_STAGE_BYTES];
  uint8_t b[STAGES][B_STAGE_BYTES];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t aux;
  uint32_t tmem_base;
  int abort;
  int tile_prefix[kMaxGroups + 1];
  int grp_start[kMaxGroups];
  int grp_rows[kMaxGroups];
  int warp_sums[kThreads / 32];
};
constexpr size_t kSmemBytes = sizeof(SmemLayout) + 1024;  // + alignment slack

struct Params {
  const int32_t* offsets;
  int offsets_plus_one;  // 1: offsets has E+1 entries starting at 0; 0: E end offsets
  int num_groups;
  int64_t m_total;       // rows of A / X / Y
  int n_out;             // output columns per tile grid (kModeRows: Nout, kModeWgrad: Q)
  int p_out;             // kModeWgrad: output rows per expert (P)
  int k_red;             // kModeRows: contraction length (Kc)
  void* out;             // kModeRows: C [m_total, n_out]; kModeWgrad: [E, p_out, n_out]
};

struct TileInfo {
  int g;       // expert
  int m_blk;   // tile row block
  int n_blk;   // tile column block
  int row0;    // kModeRows: first A row of the tile; kModeWgrad: first row of the expert
  int rows;    // kModeRows: valid output rows; kModeWgrad: rows of the expert
  int nkb;     // number of 64-wide contraction blocks
};

template <int MODE>
__device__ __forceinline__ TileInfo decode_tile(const SmemLayout& s, const Params& p, int t) {
  // Largest g with tile_prefix[g] <= t; experts that own no tile are skipped because
  // their prefix equals the next expert's.
  int lo = 0, hi = p.num_groups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s.tile_prefix[mid] <= t) lo = mid; else hi = mid - 1;
  }
  TileInfo ti;
  ti.g = lo;
  const int local = t - s.tile_prefix[lo];
  const int start = s.grp_start[lo], rows = s.grp_rows[lo];
  if (MODE == kModeRows) {
    const int mt = (rows + BM - 1) / BM;
    ti.m_blk = local % mt;
    ti.n_blk = local / mt;
    ti.row0 = start + ti.m_blk * BM;
    ti.rows = min(BM, rows - ti.m_blk * BM);
    ti.nkb = (p.k_red + BK - 1) / BK;
  } else {
    const int pt = (p.p_out + BM - 1) / BM;
    ti.m_blk = local % pt;
    ti.n_blk = local / pt;
    ti.row0 = start;
    ti.rows = rows;
    ti.nkb = (rows + BK - 1) / BK;
  }
  return ti;
}

template <int MODE>
__device__ __forceinline__ int tiles_of_group(const Params& p, int rows) {
  const int nt = (p.n_out + BN - 1) / BN;
  if (MODE == kModeRows) return ((rows + BM - 1) / BM) * nt;
  return ((p.p_out + BM - 1) / BM) * nt;
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

// A_MN / B_MN: the operand is MN-major in global memory (and in shared memory).
// In kModeRows map_b is 3-D (inner, outer, expert); every other map is 2-D (inner, row).
template <int MODE, int AB_FORMAT, bool A_MN, bool B_MN, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
gmm_sm100_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                 const Params p) {
  extern __shared__ uint8_t smem_raw[];
  SmemLayout& s = *reinterpret_cast<SmemLayout*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &s.abort;

  // ------------------------------------------------------------ prologue
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      ptx::mbar_init(ptx::smem_u32(&s.full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&s.empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(ptx::smem_u32(&s.tmem_full[i]), 1);
      ptx::mbar_init(ptx::smem_u32(&s.tmem_empty[i]), 4);
    }
    ptx::mbar_init(ptx::smem_u32(&s.aux), 1);
    s.abort = 0;
    ptx::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&map_a);
    ptx::prefetch_tensormap(&map_b);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(&s.tmem_base), kTmemCols);
    ptx::tmem_relinquish();
  }
  // Per-expert rows and tile prefix (block-wide scan; each thread owns 4 experts).
  {
    constexpr int PER = kMaxGroups / kThreads;
    const int g0 = threadIdx.x * PER;
    int cnt[PER];
    int local_sum = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int g = g0 + i;
      cnt[i] = 0;
      if (g < p.num_groups) {
        int st, en;
        if (p.offsets_plus_one) { st = p.offsets[g]; en = p.offsets[g + 1]; }
        else { st = g > 0 ? p.offsets[g - 1] : 0; en = p.offsets[g]; }
        int rows = en - st;
        if (rows < 0) rows = 0;
        s.grp_start[g] = st;
        s.grp_rows[g] = rows;
        cnt[i] = tiles_of_group<MODE>(p, rows);
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
  ptx::tc_fence_after();
  const int total_tiles = s.tile_prefix[p.num_groups];
  const uint32_t tmem_base = s.tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    int stage = 0;
    uint32_t phase = 0, aux_phase = 0;
    for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x) {
      const TileInfo ti = decode_tile<MODE>(s, p, t);
      for (int kb = 0; kb < ti.nkb; ++kb) {
        if (!ptx::wait_bounded(ptx::smem_u32(&s.empty[stage]), phase ^ 1, abort_flag,
                               kWaitTimeoutNs))
          break;
        const uint32_t sa = ptx::smem_u32(&s.a[stage][0]);
        const uint32_t sb = ptx::smem_u32(&s.b[stage][0]);
        if (MODE == kModeRows) {
          if (lane == 0) {
            const uint32_t fb = ptx::smem_u32(&s.full[stage]);
            ptx::mbar_arrive_expect_tx(fb, STAGE_BYTES);
            const int k0 = kb * BK;
            ptx::tma_load_2d(sa, &map_a, fb, k0, ti.row0);
            if (!B_MN) {
              ptx::tma_load_3d(sb, &map_b, fb, k0, ti.n_blk * BN, ti.g);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                ptx::tma_load_3d(sb + j * (BK * 128), &map_b, fb, ti.n_blk * BN + j * 64, k0, ti.g);
            }
          }
        } else {
          const int r0 = ti.row0 + kb * BK;
          const int valid = ti.row0 + ti.rows - r0;  // rows of this block inside the expert
          const bool masked = valid < BK;
          const uint32_t fb = ptx::smem_u32(&s.full[stage]);
          const uint32_t lb = masked ? ptx::smem_u32(&s.aux) : fb;
          if (lane == 0) {
            ptx::mbar_arrive_expect_tx(lb, STAGE_BYTES);
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              ptx::tma_load_2d(sa + j * (BK * 128), &map_a, lb, ti.m_blk * BM + j * 64, r0);
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              ptx::tma_load_2d(sb + j * (BK * 128), &map_b, lb, ti.n_blk * BN + j * 64, r0);
          }
          if (masked) {
            __syncwarp();
            const bool ok = ptx::wait_bounded(lb, aux_phase, abort_flag, kWaitTimeoutNs);
            aux_phase ^= 1;
            if (!ok) break;
            // Zero rows [valid, BK) of every 64-column box (2 A boxes + 4 B boxes).
            const int zrows = BK - valid;
            const int n16 = zrows * 8;  // 16-byte chunks per box
            for (int box = 0; box < (BM + BN) / 64; ++box) {
              uint8_t* base = box < BM / 64 ? &s.a[stage][box * BK * 128]
                                            : &s.b[stage][(box - BM / 64) * BK * 128];
              for (int i = lane; i < n16; i += 32) {
                reinterpret_cast<uint4*>(base + valid * 128)[i] = make_uint4(0, 0, 0, 0);
              }
            }
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(fb);
          }
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = ptx::make_idesc_f16(AB_FORMAT, A_MN ? 1 : 0, B_MN ? 1 : 0, BM, BN);
    // K-major: rows of 128 bytes, 8-row atoms 1024 bytes apart; a K=16 step is +32 bytes.
    // MN-major: 64-element column chunks BK*128 bytes apart (LBO), 8-k-row atoms 1024
    // bytes apart (SBO); a K=16 step is two atoms (+2048 bytes).
    constexpr uint32_t kLboMN = BK * 128;
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x, ++acc) {
      const TileInfo ti = decode_tile<MODE>(s, p, t);
      const int buf = acc & 1;
      const uint32_t acc_phase = (acc >> 1) & 1;
      if (!ptx::wait_bounded(ptx::smem_u32(&s.tmem_empty[buf]), acc_phase ^ 1, abort_flag,
                             kWaitTimeoutNs))
        break;
      ptx::tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * BN;
      bool ok = true;
      for (int kb = 0; kb < ti.nkb; ++kb) {
        if (!ptx::wait_bounded(ptx::smem_u32(&s.full[stage]), phase, abort_flag, kWaitTimeoutNs)) {
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
            ptx::mma_f16_ss(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          ptx::mma_commit(ptx::smem_u32(&s.empty[stage]));
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (lane == 0) {
        if (ti.nkb > 0) ptx::mma_commit(ptx::smem_u32(&s.tmem_full[buf]));
        else ptx::mbar_arrive(ptx::smem_u32(&s.tmem_full[buf]));
      }
      __syncwarp();
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;  // accumulator row owned by this thread
    OutT* out = static_cast<OutT*>(p.out);
    int acc = 0;
    for (int t = blockIdx.x; t < total_tiles && !*abort_flag; t += gridDim.x, ++acc) {
      const TileInfo ti = decode_tile<MODE>(s, p, t);
      const int buf = acc & 1;
      const uint32_t acc_phase = (acc >> 1) & 1;
      if (!ptx::wait_bounded(ptx::smem_u32(&s.tmem_full[buf]), acc_phase, abort_flag,
                             kWaitTimeoutNs))
        break;
      ptx::tc_fence_after();
      const int n0 = ti.n_blk * BN;
      const int valid_cols = min(BN, p.n_out - n0);
      int valid_rows;
      OutT* row_ptr;
      if (MODE == kModeRows) {
        valid_rows = ti.rows;
        row_ptr = out + (int64_t)(ti.row0 + r) * p.n_out + n0;
      } else {
        valid_rows = min(BM, p.p_out - ti.m_blk * BM);
        row_ptr = out + ((int64_t)ti.g * p.p_out + ti.m_blk * BM + r) * p.n_out + n0;
      }
      for (int c0 = 0; c0 < valid_cols; c0 += 32) {
        uint32_t v[32];
        if (ti.nkb > 0) {
          ptx::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN + c0, v);
          ptx::tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0u;
        }
        if (r < valid_rows) {
          if (c0 + 32 <= valid_cols) {
            if constexpr (sizeof(OutT) == 2) {
              uint4* dst = reinterpret_cast<uint4*>(row_ptr + c0);
#pragma unroll
              for (int i = 0; i < 4; ++i) dst[i] = pack8_16b<OutT>(&v[i * 8]);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) row_ptr[c0 + i] = from_f32<OutT>(__uint_as_float(v[i]));
            }
          } else {
            const int nc = valid_cols - c0;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < nc) row_ptr[c0 + i] = from_f32<OutT>(__uint_as_float(v[i]));
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&s.tmem_empty[buf]));
    }
  }

  // ------------------------------------------------------------ teardown
  __syncthreads();
  if (*abort_flag) {
    if (threadIdx.x == 0) raise_device_error(1);
    // Let any copy or MMA that was still in flight land before the memory is released.
    if (warp == 1) __nanosleep(100000);
    __syncwarp();
  }
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace gmm
}  // namespace moe
