// C ABI of the B200 MoE operator library (declarations and contracts: include/moe_b200.h).
// The library is one translation unit: this file includes every kernel header.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"
#include "ep_peer.cuh"
#include "gmm_simt.cuh"
#include "gmm_sm100.cuh"
#include "permute.cuh"
#include "swiglu.cuh"
#include "topk_softmax.cuh"

namespace moe {

static thread_local char t_err_msg[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err_msg, sizeof(t_err_msg), fmt, ap);
  va_end(ap);
  return code;
}

// Guards the per-device host-side caches (launch attributes, occupancy) that several host
// threads may fill at once.
static std::mutex g_cache_mu;

int num_sms(int device) {
  static std::atomic<int> cache[64];
  if (device >= 0 && device < 64) {
    const int c = cache[device].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
    n = 148;
  if (device >= 0 && device < 64) cache[device].store(n, std::memory_order_relaxed);
  return n;
}

static int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

// ---------------------------------------------------------------- tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 16-bit element tensor map (128-byte swizzle unless given); dims/box innermost first.
static int make_map(CUtensorMap* map, const void* base, int dtype, int rank, const uint64_t* dims,
                    const uint32_t* box,
                    CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t gdim[3], gstride[2];
  cuuint32_t bdim[3], estr[3] = {1, 1, 1};
  uint64_t stride = 2;
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    if (i > 0) gstride[i - 1] = stride;
    stride *= dims[i];
  }
  const CUtensorMapDataType dt =
      dtype == MOE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, (cuuint32_t)rank, const_cast<void*>(base), gdim, gstride, bdim, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rank=%d dims=%llu,%llu,%llu",
                     (int)r, rank, (unsigned long long)dims[0],
                     (unsigned long long)(rank > 1 ? dims[1] : 0),
                     (unsigned long long)(rank > 2 ? dims[2] : 0));
  return MOE_OK;
}

// ---------------------------------------------------------------- GEMM launchers
template <int MODE, int CG, int FMT, bool A_MN, bool B_MN, typename OutT>
// `extra` (kModeGateUp): the up-projection weights' map, then the gate and up output maps.
static int launch_sm100(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                        const gmm::Params& p, cudaStream_t stream,
                        const CUtensorMap* extra = nullptr) {
  auto kern = gmm::gmm_sm100_kernel<MODE, CG, FMT, A_MN, B_MN, OutT>;
  const int dev = current_device();
  static unsigned long long attr_set = 0;  // per-device bitmask, one per instantiation
  static int max_clusters[64] = {0};
  {
    std::lock_guard<std::mutex> lock(g_cache_mu);
    if (dev < 64 && !(attr_set & (1ull << dev))) {
      MOE_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)gmm::smem_bytes<CG>()));
      attr_set |= 1ull << dev;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(gmm::kThreads);
  cfg.dynamicSmemBytes = gmm::smem_bytes<CG>();
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = CG == 2 ? 1 : 0;
  // A persistent kernel strides tiles statically, so every CTA must be resident at once:
  // for SM pairs the grid is the number of clusters that fit together (cluster placement
  // is per GPC, so it can be below #SMs / 2).
  int grid = (num_sms(dev) / CG) * CG;
  if (CG == 2 && dev < 64) {
    std::lock_guard<std::mutex> lock(g_cache_mu);
    if (max_clusters[dev] == 0) {
      cfg.gridDim = dim3(grid);
      int n = 0;
      MOE_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
      max_clusters[dev] = n > 0 ? n : 1;
    }
    grid = std::min(grid, max_clusters[dev] * CG);
  }
  cfg.gridDim = dim3(grid);
  if (getenv("MOE_B200_DEBUG"))
    fprintf(stderr, "[moe_b200] gmm launch: mode=%d cg=%d grid=%d smem=%zu\n", MODE, CG, grid,
            gmm::smem_bytes<CG>());
  MOE_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, extra ? extra[0] : mb,
                                    extra ? extra[1] : mc, extra ? extra[2] : mc, p));
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

// Launch with programmatic stream serialization: the kernel may start before the previous
// kernel of the stream completes and waits for it with pdl_wait() (hides launch latency in
// chains of short kernels).
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// The unpermute-forward kernel for a row set R: the vector path instantiated for the
// smallest KMAX >= topk (all K slots' loads in flight together), the element path once.
#define MOE_UNP_LAUNCH(TT, PP, R)                                                                   \
  if (vec) {                                                                                        \
    if (topk <= 2)                                                                                  \
      unpermute_fwd_kernel<TT, PP, 2, true><<<grid, kRowWarps * 32, 0, s>>>(                        \
          R, (const PP*)prob, (TT*)out, num_tokens, topk, num_cols);                                \
    else if (topk <= 4)                                                                             \
      unpermute_fwd_kernel<TT, PP, 4, true><<<grid, kRowWarps * 32, 0, s>>>(                        \
          R, (const PP*)prob, (TT*)out, num_tokens, topk, num_cols);                                \
    else if (topk <= 8)                                                                             \
      unpermute_fwd_kernel<TT, PP, 8, true><<<grid, kRowWarps * 32, 0, s>>>(                        \
          R, (const PP*)prob, (TT*)out, num_tokens, topk, num_cols);                                \
    else                                                                                            \
      unpermute_fwd_kernel<TT, PP, 32, true><<<grid, kRowWarps * 32, 0, s>>>(                       \
          R, (const PP*)prob, (TT*)out, num_tokens, topk, num_cols);                                \
  } else {                                                                                          \
    unpermute_fwd_kernel<TT, PP, 32, false><<<grid, kRowWarps * 32, 0, s>>>(                        \
        R, (const PP*)prob, (TT*)out, num_tokens, topk, num_cols);                                  \
  }

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// CTA-group choice: MOE_B200_GMM_CG=1|2 forces it (tuning/tests); otherwise `auto_cg`.
static int pick_cg(int auto_cg) {
  const char* e = getenv("MOE_B200_GMM_CG");
  return (e && (e[0] == '1' || e[0] == '2') && e[1] == 0) ? e[0] - '0' : auto_cg;
}

template <int MODE, bool A_MN, bool B_MN>
static int launch_fmt_cg(int dtype, int cg, const CUtensorMap& ma, const CUtensorMap& mb,
                         const CUtensorMap& mc, const gmm::Params& p, cudaStream_t stream) {
  if (dtype == MOE_BF16)
    return cg == 2 ? launch_sm100<MODE, 2, 1, A_MN, B_MN, __nv_bfloat16>(ma, mb, mc, p, stream)
                   : launch_sm100<MODE, 1, 1, A_MN, B_MN, __nv_bfloat16>(ma, mb, mc, p, stream);
  return cg == 2 ? launch_sm100<MODE, 2, 0, A_MN, B_MN, __half>(ma, mb, mc, p, stream)
                 : launch_sm100<MODE, 1, 0, A_MN, B_MN, __half>(ma, mb, mc, p, stream);
}

// SwiGLU backward applied to a row-mode product D (the gradient of h = silu(gate) * up):
// C receives the gradient of gate, grad_up that of up.
struct SwiGLUBwdArgs {
  const void* gate;
  const void* up;
  void* grad_up;
};

static int swiglu_bwd_launch(const void* grad_out, const void* gate, const void* up,
                             void* grad_gate, void* grad_up, int64_t n, int dtype,
                             cudaStream_t s);

// Row mode (forward / dgrad): C[m_total, n_out] = A[m_total, k_red] . op(B[g]).
// b_mn: B[g] stored [k_red, n_out] (MN-major) instead of [n_out, k_red].
// sw: also apply the SwiGLU backward to the product (C becomes the gate gradient).
// seg2: a second contraction segment into the same accumulator, C = A . op(B[g]) +
// seg2->A . op(seg2->B[g]) (tensor-core path only; the caller checks gmm_rows_dual_ok).
struct RowsSeg2 {
  const void* A;
  const void* B;
  int64_t k_red;
};

// A gathered operand: row r is row rows[r] of a [src_rows, ...] tensor (TMA gather4).
struct GatherArgs {
  const int32_t* rows;
  int64_t src_rows;
};

static int gmm_rows(const void* A, const void* B, void* C, const int32_t* offsets, int plus_one,
                    int64_t m_total, int64_t n_out, int64_t k_red, int E, bool b_mn, int dtype,
                    cudaStream_t stream, const SwiGLUBwdArgs* sw = nullptr,
                    const RowsSeg2* seg2 = nullptr, const GatherArgs* ga = nullptr) {
  if (m_total == 0 || n_out == 0) return MOE_OK;
  const bool tc = dtype != MOE_F32 && k_red % 8 == 0 && n_out % 8 == 0 && E <= gmm::kMaxGroups &&
                  aligned16(A) && aligned16(B) && aligned16(C) && m_total < (1ll << 31) &&
                  n_out < (1ll << 31) && k_red < (1ll << 31) &&
                  (!sw || (aligned16(sw->gate) && aligned16(sw->up) && aligned16(sw->grad_up)));
  if (ga) {
    MOE_REQUIRE(tc && k_red > 0 && !sw && !seg2 && ga->rows != nullptr && ga->src_rows > 0 &&
                    ga->src_rows < (1ll << 31),
                "gmm gather: needs the tensor-core path (16-bit, aligned, sizes multiples of 8)");
  }
  if (sw && (!tc || k_red == 0)) {
    // The product into C, then the SwiGLU backward in place (each element is read before
    // the same thread writes it).
    int rc = gmm_rows(A, B, C, offsets, plus_one, m_total, n_out, k_red, E, b_mn, dtype, stream);
    if (rc) return rc;
    return swiglu_bwd_launch(C, sw->gate, sw->up, C, sw->grad_up, m_total * n_out, dtype, stream);
  }
  if (!tc || k_red == 0) {
    if (k_red == 0) {
      MOE_CUDA_CHECK(cudaMemsetAsync(C, 0, (size_t)m_total * n_out * dtype_size(dtype), stream));
      return MOE_OK;
    }
    const dim3 grid((unsigned)((m_total + simt::TM - 1) / simt::TM),
                    (unsigned)((n_out + simt::TN - 1) / simt::TN), (unsigned)E);
    MOE_REQUIRE(grid.y <= 65535 && grid.z <= 65535, "gmm: grid too large for the CUDA-core path");
    switch (dtype) {
      case MOE_F32:
        simt::gmm_rows_simt_kernel<float><<<grid, 256, 0, stream>>>(
            (const float*)A, (const float*)B, (float*)C, offsets, plus_one, n_out, k_red, b_mn);
        break;
      case MOE_F16:
        simt::gmm_rows_simt_kernel<__half><<<grid, 256, 0, stream>>>(
            (const __half*)A, (const __half*)B, (__half*)C, offsets, plus_one, n_out, k_red, b_mn);
        break;
      default:
        simt::gmm_rows_simt_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
            (const __nv_bfloat16*)A, (const __nv_bfloat16*)B, (__nv_bfloat16*)C, offsets,
            plus_one, n_out, k_red, b_mn);
    }
    MOE_LAUNCH_CHECK();
    return MOE_OK;
  }
  // SM pairs once experts average 1024 rows or more (measured, cfg2 d=4096: dgrad 1290 vs
  // 1237 TFLOP/s, forward even); single CTAs below (cfg4's 256 rows: forward 956 vs 916).
  const int cg = (sw || seg2 || ga) ? 1 : pick_cg(m_total >= 1024ll * E ? 2 : 1);
  const uint32_t b_cols = (uint32_t)(gmm::BN / cg);
  CUtensorMap ma, mb;
  {
    // 64-row boxes: two per CTA, one per CTA of a half tile; a gathered A: one-row boxes
    // over the source rows.
    const uint64_t dims[2] = {(uint64_t)k_red, (uint64_t)(ga ? ga->src_rows : m_total)};
    const uint32_t box[2] = {(uint32_t)gmm::BK, ga ? 1u : 64u};
    int rc = make_map(&ma, A, dtype, 2, dims, box);
    if (rc) return rc;
  }
  if (!b_mn) {
    const uint64_t dims[3] = {(uint64_t)k_red, (uint64_t)n_out, (uint64_t)E};
    const uint32_t box[3] = {(uint32_t)gmm::BK, b_cols, 1};
    int rc = make_map(&mb, B, dtype, 3, dims, box);
    if (rc) return rc;
  } else {
    const uint64_t dims[3] = {(uint64_t)n_out, (uint64_t)k_red, (uint64_t)E};
    const uint32_t box[3] = {64, (uint32_t)gmm::BK, 1};
    int rc = make_map(&mb, B, dtype, 3, dims, box);
    if (rc) return rc;
  }
  CUtensorMap ma2, mb2;  // second segment: A2 [m_total, k_red2], B2 like B
  if (seg2) {
    const uint64_t dims[2] = {(uint64_t)seg2->k_red, (uint64_t)m_total};
    const uint32_t box[2] = {(uint32_t)gmm::BK, 64u};
    int rc = make_map(&ma2, seg2->A, dtype, 2, dims, box);
    if (rc) return rc;
    if (!b_mn) {
      const uint64_t d3[3] = {(uint64_t)seg2->k_red, (uint64_t)n_out, (uint64_t)E};
      const uint32_t b3[3] = {(uint32_t)gmm::BK, b_cols, 1};
      rc = make_map(&mb2, seg2->B, dtype, 3, d3, b3);
    } else {
      const uint64_t d3[3] = {(uint64_t)n_out, (uint64_t)seg2->k_red, (uint64_t)E};
      const uint32_t b3[3] = {64, (uint32_t)gmm::BK, 1};
      rc = make_map(&mb2, seg2->B, dtype, 3, d3, b3);
    }
    if (rc) return rc;
  }
  CUtensorMap mc, mc_up;  // outputs, 32 x 32 boxes in the epilogue's 64-byte swizzle
  {
    const uint64_t dims[2] = {(uint64_t)n_out, (uint64_t)m_total};
    const uint32_t box[2] = {32, 32};
    int rc = make_map(&mc, C, dtype, 2, dims, box, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
    if (sw && (rc = make_map(&mc_up, sw->grad_up, dtype, 2, dims, box, CU_TENSOR_MAP_SWIZZLE_64B)))
      return rc;
  }
  gmm::Params p = {};
  p.offsets = offsets;
  p.offsets_plus_one = plus_one;
  p.num_groups = E;
  p.m_total = m_total;
  p.n_out = (int)n_out;
  p.p_out = 0;
  p.k_red = (int)k_red;
  p.out = C;
  if (ga) {
    p.gather_rows = ga->rows;
    p.gather_src_rows = (int)ga->src_rows;
  }
  if (sw) {
    p.out_up = sw->grad_up;
    p.in_gate = sw->gate;
    p.in_up = sw->up;
    const CUtensorMap extra[3] = {mb, mc, mc_up};
    constexpr int M3 = gmm::kModeSwiGLUBwd;
    if (dtype == MOE_BF16)
      return b_mn ? launch_sm100<M3, 1, 1, false, true, __nv_bfloat16>(ma, mb, mc, p, stream, extra)
                  : launch_sm100<M3, 1, 1, false, false, __nv_bfloat16>(ma, mb, mc, p, stream, extra);
    return b_mn ? launch_sm100<M3, 1, 0, false, true, __half>(ma, mb, mc, p, stream, extra)
                : launch_sm100<M3, 1, 0, false, false, __half>(ma, mb, mc, p, stream, extra);
  }
  if (seg2) {
    // map_b2 carries B2 and map_c2 carries A2 (row mode stores through map_c only).
    p.k_red2 = (int)seg2->k_red;
    const CUtensorMap extra[3] = {mb2, ma2, mc};
    if (dtype == MOE_BF16)
      return b_mn ? launch_sm100<gmm::kModeRows, 1, 1, false, true, __nv_bfloat16>(ma, mb, mc, p, stream, extra)
                  : launch_sm100<gmm::kModeRows, 1, 1, false, false, __nv_bfloat16>(ma, mb, mc, p, stream, extra);
    return b_mn ? launch_sm100<gmm::kModeRows, 1, 0, false, true, __half>(ma, mb, mc, p, stream, extra)
                : launch_sm100<gmm::kModeRows, 1, 0, false, false, __half>(ma, mb, mc, p, stream, extra);
  }
  return b_mn ? launch_fmt_cg<gmm::kModeRows, false, true>(dtype, cg, ma, mb, mc, p, stream)
              : launch_fmt_cg<gmm::kModeRows, false, false>(dtype, cg, ma, mb, mc, p, stream);
}

// Wgrad mode: Out[g] [P, Q] = X[rows of g]^T . Y[rows of g]; X [m_total, P], Y [m_total, Q].
static int gmm_wgrad(const void* X, const void* Y, void* Out, const int32_t* offsets, int plus_one,
                     int64_t m_total, int64_t P, int64_t Q, int E, int dtype, cudaStream_t stream,
                     const GatherArgs* ga = nullptr) {
  if (P == 0 || Q == 0 || E == 0) return MOE_OK;
  const bool tc = dtype != MOE_F32 && P % 8 == 0 && Q % 8 == 0 && E <= gmm::kMaxGroups &&
                  aligned16(X) && aligned16(Y) && aligned16(Out) && m_total > 0 &&
                  m_total < (1ll << 31) && P < (1ll << 31) && Q < (1ll << 31);
  if (ga) {
    MOE_REQUIRE(tc && ga->rows != nullptr && ga->src_rows > 0 && ga->src_rows < (1ll << 31),
                "gmm wgrad gather: needs the tensor-core path (16-bit, aligned, sizes multiples of 8)");
  }
  if (!tc) {
    const dim3 grid((unsigned)((Q + simt::TN - 1) / simt::TN), (unsigned)((P + simt::TM - 1) / simt::TM),
                    (unsigned)E);
    MOE_REQUIRE(grid.y <= 65535 && grid.z <= 65535, "gmm wgrad: grid too large for the CUDA-core path");
    switch (dtype) {
      case MOE_F32:
        simt::gmm_wgrad_simt_kernel<float><<<grid, 256, 0, stream>>>(
            (const float*)X, (const float*)Y, (float*)Out, offsets, plus_one, P, Q);
        break;
      case MOE_F16:
        simt::gmm_wgrad_simt_kernel<__half><<<grid, 256, 0, stream>>>(
            (const __half*)X, (const __half*)Y, (__half*)Out, offsets, plus_one, P, Q);
        break;
      default:
        simt::gmm_wgrad_simt_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
            (const __nv_bfloat16*)X, (const __nv_bfloat16*)Y, (__nv_bfloat16*)Out, offsets,
            plus_one, P, Q);
    }
    MOE_LAUNCH_CHECK();
    return MOE_OK;
  }
  const int cg = pick_cg(P > gmm::BMC ? 2 : 1);
  CUtensorMap mx, my;
  {
    const uint64_t dims[2] = {(uint64_t)P, (uint64_t)m_total};
    const uint32_t box[2] = {64, (uint32_t)gmm::BK};
    int rc = make_map(&mx, X, dtype, 2, dims, box);
    if (rc) return rc;
  }
  {
    // A gathered Y: one-row boxes over the source rows.
    const uint64_t dims[2] = {(uint64_t)Q, (uint64_t)(ga ? ga->src_rows : m_total)};
    const uint32_t box[2] = {64, ga ? 1u : (uint32_t)gmm::BK};
    int rc = make_map(&my, Y, dtype, 2, dims, box);
    if (rc) return rc;
  }
  CUtensorMap mo;  // output [E, P, Q], 32 x 32 boxes in the epilogue's 64-byte swizzle
  {
    const uint64_t dims[3] = {(uint64_t)Q, (uint64_t)P, (uint64_t)E};
    const uint32_t box[3] = {32, 32, 1};
    int rc = make_map(&mo, Out, dtype, 3, dims, box, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
  }
  gmm::Params p = {};
  p.offsets = offsets;
  p.offsets_plus_one = plus_one;
  p.num_groups = E;
  p.m_total = m_total;
  p.n_out = (int)Q;
  p.p_out = (int)P;
  p.k_red = 0;
  p.out = Out;
  {
    const char* e = getenv("MOE_B200_WGRAD_ORDER");  // tuning: p = row blocks fastest
    p.q_fastest = (e && e[0] == 'p') ? 0 : 1;
  }
  if (ga) {
    p.gather_rows = ga->rows;
    p.gather_src_rows = (int)ga->src_rows;
  }
  return launch_fmt_cg<gmm::kModeWgrad, true, true>(dtype, cg, mx, my, mo, p, stream);
}

static int check_gmm_args(const void* a, const void* b, const void* c, const int32_t* offsets,
                          int num_offsets, int64_t m_total, int64_t n, int64_t k, int E, int dtype) {
  MOE_REQUIRE(dtype_ok(dtype), "gmm: bad dtype %d", dtype);
  MOE_REQUIRE(E >= 0 && m_total >= 0 && n >= 0 && k >= 0, "gmm: negative size");
  MOE_REQUIRE(num_offsets == E || num_offsets == E + 1,
              "gmm: num_offsets must be E or E+1 (got %d, E=%d)", num_offsets, E);
  MOE_REQUIRE(E == 0 || offsets != nullptr, "gmm: offsets is NULL");
  MOE_REQUIRE((a && b && c) || m_total == 0 || E == 0, "gmm: NULL operand");
  return MOE_OK;
}

// ---------------------------------------------------------------- permute workspace
// Workspace: cnt[E][num_tiles] int32.
struct PermuteWorkspace {
  int64_t num_tiles;
  size_t cnt_bytes;
  size_t total_bytes;
};
static PermuteWorkspace permute_ws(int64_t T, int K, int E) {
  PermuteWorkspace w;
  w.num_tiles = permute_num_tiles(T * (int64_t)K);
  w.cnt_bytes = (size_t)w.num_tiles * E * sizeof(int32_t);
  w.total_bytes = w.cnt_bytes + 16;
  return w;
}

// Zero fill with 16-byte stores (the write-bandwidth probe).
__global__ void __launch_bounds__(256) write_probe_kernel(uint4* __restrict__ p, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    p[i] = make_uint4(0, 0, 0, 0);
}

// Grid of the grid-stride elementwise kernels: up to 8 blocks of 256 threads per SM.
static unsigned elementwise_grid(int64_t n, int per_thread) {
  const int64_t blocks = (n / per_thread + 255) / 256;
  const int64_t cap = (int64_t)num_sms(current_device()) * 8;
  return (unsigned)std::max<int64_t>(1, std::min(blocks, cap));
}

static int swiglu_bwd_launch(const void* grad_out, const void* gate, const void* up,
                             void* grad_gate, void* grad_up, int64_t n, int dtype,
                             cudaStream_t s) {
  if (n == 0) return MOE_OK;
  const unsigned grid = elementwise_grid(n, 16 / dtype_size(dtype));
  switch (dtype) {
    case MOE_F32: swiglu_bwd_kernel<float><<<grid, 256, 0, s>>>((const float*)grad_out, (const float*)gate, (const float*)up, (float*)grad_gate, (float*)grad_up, n); break;
    case MOE_F16: swiglu_bwd_kernel<__half><<<grid, 256, 0, s>>>((const __half*)grad_out, (const __half*)gate, (const __half*)up, (__half*)grad_gate, (__half*)grad_up, n); break;
    default: swiglu_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)grad_out, (const __nv_bfloat16*)gate, (const __nv_bfloat16*)up, (__nv_bfloat16*)grad_gate, (__nv_bfloat16*)grad_up, n);
  }
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

}  // namespace moe

using namespace moe;

extern "C" {

const char* moe_version(void) { return "moe_b200 0.1.0 sm_100a"; }

const char* moe_last_error_string(void) { return t_err_msg; }

int moe_read_device_error(int* code_out) {
  int v = 0, zero = 0;
  MOE_CUDA_CHECK(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  MOE_CUDA_CHECK(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  if (code_out) *code_out = v;
  return MOE_OK;
}

int moe_peek_device_error(void* dst, void* stream) {
  MOE_REQUIRE(dst != nullptr, "peek_device_error: dst is NULL");
  MOE_CUDA_CHECK(cudaMemcpyFromSymbolAsync(dst, g_device_error, sizeof(int), 0, cudaMemcpyDefault,
                                           (cudaStream_t)stream));
  return MOE_OK;
}

int moe_topk_softmax_fwd(const void* logits, int dtype, int64_t num_tokens, int32_t E, int32_t K,
                         void* weights, int32_t* indices, void* stream) {
  MOE_REQUIRE(dtype_ok(dtype), "topk_softmax: bad dtype %d", dtype);
  MOE_REQUIRE(num_tokens >= 0 && E > 0 && K > 0 && K <= E && K <= 32,
              "topk_softmax: need 0 < K <= min(E, 32) (E=%d, K=%d)", E, K);
  if (num_tokens == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  switch (dtype) {
    case MOE_F32: return launch_topk_fwd<float>(logits, num_tokens, E, K, weights, indices, s);
    case MOE_F16: return launch_topk_fwd<__half>(logits, num_tokens, E, K, weights, indices, s);
    default: return launch_topk_fwd<__nv_bfloat16>(logits, num_tokens, E, K, weights, indices, s);
  }
}

int moe_topk_softmax_bwd(const void* grad_weights, const void* weights, const int32_t* indices,
                         int dtype, int64_t num_tokens, int32_t E, int32_t K, void* grad_logits,
                         void* stream) {
  MOE_REQUIRE(dtype_ok(dtype), "topk_softmax_bwd: bad dtype %d", dtype);
  MOE_REQUIRE(num_tokens >= 0 && E > 0 && K > 0 && K <= 32, "topk_softmax_bwd: bad E=%d K=%d", E, K);
  if (num_tokens == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  switch (dtype) {
    case MOE_F32: return launch_topk_bwd<float>(grad_weights, weights, indices, num_tokens, E, K, grad_logits, s);
    case MOE_F16: return launch_topk_bwd<__half>(grad_weights, weights, indices, num_tokens, E, K, grad_logits, s);
    default: return launch_topk_bwd<__nv_bfloat16>(grad_weights, weights, indices, num_tokens, E, K, grad_logits, s);
  }
}

size_t moe_permute_workspace_bytes(int64_t num_tokens, int32_t topk, int32_t E) {
  if (num_tokens <= 0 || topk <= 0 || E <= 0) return 16;
  return permute_ws(num_tokens, topk, E).total_bytes;
}

}  // extern "C"

namespace moe {
// The counting-sort permute with optional dropping (see permute_rank_kernel): a slot is
// kept while its rank inside its expert is below `capacity` and its row below `row_limit`.
static int permute_impl(const void* input, int dtype, const int32_t* indices, int64_t num_tokens,
                        int32_t topk, int64_t num_cols, int32_t E, int32_t capacity,
                        int32_t row_limit, void* permuted, int32_t* row_id_map, int32_t* offsets,
                        void* workspace, size_t workspace_bytes, void* stream,
                        int32_t* row_src = nullptr) {
  const int64_t num_slots = num_tokens * topk;
  cudaStream_t s = (cudaStream_t)stream;
  if (num_slots == 0) {
    MOE_CUDA_CHECK(cudaMemsetAsync(offsets, 0, (E + 1) * sizeof(int32_t), s));
    return MOE_OK;
  }
  const PermuteWorkspace w = permute_ws(num_tokens, topk, E);
  if (workspace == nullptr || workspace_bytes < w.total_bytes)
    return set_error(MOE_ERR_WORKSPACE, "permute: workspace needs %zu bytes (got %zu)",
                     w.total_bytes, workspace_bytes);
  int32_t* cnt = static_cast<int32_t*>(workspace);
  const unsigned tiles = (unsigned)w.num_tiles;
  permute_hist_kernel<<<tiles, kPermTile, E * sizeof(int32_t), s>>>(indices, num_slots, E, cnt,
                                                                     w.num_tiles);
  MOE_LAUNCH_CHECK();
  const size_t rank_smem = (size_t)(kPermTileWarps + 3) * E * sizeof(int32_t);
  if (rank_smem > 48 * 1024) {
    // The opt-in limit only grows, so a concurrent call with a smaller E never lowers it
    // under a launch that needs more.
    static size_t rank_smem_set[64] = {0};
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(g_cache_mu);
    if (dev >= 64 || rank_smem > rank_smem_set[dev]) {
      MOE_CUDA_CHECK(cudaFuncSetAttribute(permute_rank_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)rank_smem));
      if (dev < 64) rank_smem_set[dev] = rank_smem;
    }
  }
  MOE_CUDA_CHECK(launch_pdl(permute_rank_kernel, dim3(tiles), dim3(kPermTile), rank_smem, s, indices,
                            num_slots, num_tokens, topk, E, (const int32_t*)cnt, w.num_tiles,
                            row_id_map, offsets, capacity, row_limit, row_src));
  if (num_cols == 0) return MOE_OK;
  const int es = dtype_size(dtype);
  const bool vec = (num_cols * es) % 16 == 0 && aligned16(input) && aligned16(permuted);
  const dim3 grid((unsigned)((num_tokens + kRowWarps - 1) / kRowWarps));
#define MOE_COPY(TT)                                                                                 \
  {                                                                                                 \
    const LocalRows<TT> rows{(TT*)permuted, row_id_map, num_tokens, num_cols};                      \
    if (vec)                                                                                        \
      MOE_CUDA_CHECK(launch_pdl(permute_copy_kernel<TT, true, LocalRows<TT>>, grid,                 \
                                dim3(kRowWarps * 32), 0, s, (const TT*)input, rows, num_tokens,     \
                                topk, num_cols));                                                  \
    else                                                                                            \
      MOE_CUDA_CHECK(launch_pdl(permute_copy_kernel<TT, false, LocalRows<TT>>, grid,                \
                                dim3(kRowWarps * 32), 0, s, (const TT*)input, rows, num_tokens,     \
                                topk, num_cols));                                                  \
  }
  switch (dtype) {
    case MOE_F32: MOE_COPY(float) break;
    case MOE_F16: MOE_COPY(__half) break;
    default: MOE_COPY(__nv_bfloat16) break;
  }
#undef MOE_COPY
  return MOE_OK;
}
}  // namespace moe

extern "C" {

int moe_permute(const void* input, int dtype, const int32_t* indices, int64_t num_tokens,
                int32_t topk, int64_t num_cols, int32_t E, int64_t num_out, void* permuted,
                int32_t* row_id_map, int32_t* offsets, void* workspace, size_t workspace_bytes,
                void* stream) {
  MOE_REQUIRE(dtype_ok(dtype), "permute: bad dtype %d", dtype);
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && topk <= 32 && num_cols >= 0,
              "permute: bad sizes T=%lld K=%d C=%lld", (long long)num_tokens, topk, (long long)num_cols);
  MOE_REQUIRE(E > 0 && E <= kMaxExperts, "permute: need 0 < E <= %d (E=%d)", kMaxExperts, E);
  const int64_t num_slots = num_tokens * topk;
  MOE_REQUIRE(num_out >= num_slots, "permute: num_out (%lld) < T*K (%lld)", (long long)num_out,
              (long long)num_slots);
  MOE_REQUIRE(num_slots < (1ll << 31), "permute: T*K must fit in int32");
  return permute_impl(input, dtype, indices, num_tokens, topk, num_cols, E, INT32_MAX, INT32_MAX,
                      permuted, row_id_map, offsets, workspace, workspace_bytes, stream);
}

int moe_permute_index(const int32_t* indices, int64_t num_tokens, int32_t topk, int32_t E,
                      int32_t* row_id_map, int32_t* offsets, int32_t* row_src, void* workspace,
                      size_t workspace_bytes, void* stream) {
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && topk <= 32, "permute_index: bad sizes T=%lld K=%d",
              (long long)num_tokens, topk);
  MOE_REQUIRE(E > 0 && E <= kMaxExperts, "permute_index: need 0 < E <= %d (E=%d)", kMaxExperts, E);
  MOE_REQUIRE(num_tokens * topk < (1ll << 31), "permute_index: T*K must fit in int32");
  MOE_REQUIRE(row_src != nullptr, "permute_index: row_src is NULL");
  return permute_impl(nullptr, MOE_BF16, indices, num_tokens, topk, 0, E, INT32_MAX, INT32_MAX,
                      nullptr, row_id_map, offsets, workspace, workspace_bytes, stream, row_src);
}

int moe_permute_capacity(const void* input, int dtype, const int32_t* indices, int64_t num_tokens,
                         int32_t topk, int64_t num_cols, int32_t E, int32_t capacity,
                         int64_t num_out, void* permuted, int32_t* row_id_map, int32_t* offsets,
                         void* workspace, size_t workspace_bytes, void* stream) {
  MOE_REQUIRE(dtype_ok(dtype), "permute_capacity: bad dtype %d", dtype);
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && topk <= 32 && num_cols >= 0,
              "permute_capacity: bad sizes T=%lld K=%d C=%lld", (long long)num_tokens, topk,
              (long long)num_cols);
  MOE_REQUIRE(E > 0 && E <= kMaxExperts, "permute_capacity: need 0 < E <= %d (E=%d)", kMaxExperts, E);
  const int64_t num_slots = num_tokens * topk;
  MOE_REQUIRE(num_slots < (1ll << 31), "permute_capacity: T*K must fit in int32");
  MOE_REQUIRE(num_out >= 0 && num_out < (1ll << 31), "permute_capacity: bad num_out %lld",
              (long long)num_out);
  return permute_impl(input, dtype, indices, num_tokens, topk, num_cols, E,
                      capacity > 0 ? capacity : INT32_MAX, (int32_t)num_out, permuted, row_id_map,
                      offsets, workspace, workspace_bytes, stream);
}

int moe_swiglu_fwd(const void* gate, const void* up, void* out, int64_t n, int dtype, void* stream) {
  MOE_REQUIRE(dtype == MOE_BF16 || dtype == MOE_F16 || dtype == MOE_F32, "swiglu: bad dtype %d", dtype);
  MOE_REQUIRE(n >= 0, "swiglu: negative size");
  MOE_REQUIRE(aligned16(gate) && aligned16(up) && aligned16(out), "swiglu: pointers must be 16-byte aligned");
  if (n == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned grid = elementwise_grid(n, 16 / dtype_size(dtype));
  switch (dtype) {
    case MOE_F32: swiglu_fwd_kernel<float><<<grid, 256, 0, s>>>((const float*)gate, (const float*)up, (float*)out, n); break;
    case MOE_F16: swiglu_fwd_kernel<__half><<<grid, 256, 0, s>>>((const __half*)gate, (const __half*)up, (__half*)out, n); break;
    default: swiglu_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)gate, (const __nv_bfloat16*)up, (__nv_bfloat16*)out, n);
  }
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_swiglu_bwd(const void* grad_out, const void* gate, const void* up, void* grad_gate,
                   void* grad_up, int64_t n, int dtype, void* stream) {
  MOE_REQUIRE(dtype == MOE_BF16 || dtype == MOE_F16 || dtype == MOE_F32, "swiglu_bwd: bad dtype %d", dtype);
  MOE_REQUIRE(n >= 0, "swiglu_bwd: negative size");
  MOE_REQUIRE(aligned16(grad_out) && aligned16(gate) && aligned16(up) && aligned16(grad_gate) &&
                  aligned16(grad_up),
              "swiglu_bwd: pointers must be 16-byte aligned");
  return swiglu_bwd_launch(grad_out, gate, up, grad_gate, grad_up, n, dtype, (cudaStream_t)stream);
}

int moe_scatter_rows(const void* input, int dtype, const int32_t* row_id_map, int64_t num_tokens,
                     int32_t topk, int64_t num_cols, void* out, void* stream) {
  MOE_REQUIRE(dtype_ok(dtype), "scatter_rows: bad dtype %d", dtype);
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && topk <= 32 && num_cols >= 0, "scatter_rows: bad sizes");
  if (num_tokens == 0 || num_cols == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const bool vec = (num_cols * dtype_size(dtype)) % 16 == 0 && aligned16(input) && aligned16(out);
  const dim3 grid((unsigned)((num_tokens + kRowWarps - 1) / kRowWarps));
#define MOE_SC(TT)                                                                                   \
  {                                                                                                 \
    const LocalRows<TT> rows{(TT*)out, row_id_map, num_tokens, num_cols};                           \
    if (vec)                                                                                        \
      permute_copy_kernel<TT, true><<<grid, kRowWarps * 32, 0, s>>>((const TT*)input, rows,          \
                                                                    num_tokens, topk, num_cols);   \
    else                                                                                            \
      permute_copy_kernel<TT, false><<<grid, kRowWarps * 32, 0, s>>>((const TT*)input, rows,         \
                                                                     num_tokens, topk, num_cols);  \
  }
  switch (dtype) {
    case MOE_F32: MOE_SC(float) break;
    case MOE_F16: MOE_SC(__half) break;
    default: MOE_SC(__nv_bfloat16) break;
  }
#undef MOE_SC
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_unpermute_fwd(const void* input, int dtype, const int32_t* row_id_map, const void* prob,
                      int prob_dtype, int64_t num_tokens, int32_t topk, int64_t num_cols, void* out,
                      void* stream) {
  MOE_REQUIRE(dtype_ok(dtype) && (prob == nullptr || dtype_ok(prob_dtype)),
              "unpermute: bad dtype %d / prob dtype %d", dtype, prob_dtype);
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && topk <= 32 && num_cols >= 0, "unpermute: bad sizes");
  if (num_tokens == 0 || num_cols == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int es = dtype_size(dtype);
  const bool vec = (num_cols * es) % 16 == 0 && aligned16(input) && aligned16(out);
  const dim3 grid((unsigned)((num_tokens + kRowWarps - 1) / kRowWarps));
  const int pd = prob == nullptr ? MOE_F32 : prob_dtype;
#define MOE_UNP(TT, PP)                                                                              \
  {                                                                                                 \
    const LocalRows<const TT> rows{(const TT*)input, row_id_map, num_tokens, num_cols};             \
    MOE_UNP_LAUNCH(TT, PP, rows)                                                                    \
  }
#define MOE_UNP_P(TT)                                                                                \
  switch (pd) {                                                                                     \
    case MOE_F32: MOE_UNP(TT, float) break;                                                         \
    case MOE_F16: MOE_UNP(TT, __half) break;                                                        \
    default: MOE_UNP(TT, __nv_bfloat16) break;                                                      \
  }
  switch (dtype) {
    case MOE_F32: MOE_UNP_P(float) break;
    case MOE_F16: MOE_UNP_P(__half) break;
    default: MOE_UNP_P(__nv_bfloat16) break;
  }
#undef MOE_UNP_P
#undef MOE_UNP
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_unpermute_bwd(const void* grad_out, const void* input_fwd, int dtype,
                      const int32_t* row_id_map, const void* prob, int prob_dtype,
                      int64_t num_tokens, int32_t topk, int64_t num_cols, void* act_grad,
                      void* prob_grad, void* stream) {
  MOE_REQUIRE(dtype_ok(dtype) && dtype_ok(prob_dtype), "unpermute_bwd: bad dtype");
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && topk <= 32 && num_cols >= 0, "unpermute_bwd: bad sizes");
  MOE_REQUIRE(prob != nullptr && prob_grad != nullptr, "unpermute_bwd: prob / prob_grad is NULL");
  if (num_tokens == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int es = dtype_size(dtype);
  const bool vec = (num_cols * es) % 16 == 0 && aligned16(grad_out) && aligned16(input_fwd) &&
                   aligned16(act_grad);
  const dim3 grid((unsigned)((num_tokens + kRowWarps - 1) / kRowWarps));
#define MOE_UB(TT, PP, KM)                                                                           \
  {                                                                                                 \
    const LocalRows<const TT> in_rows{(const TT*)input_fwd, row_id_map, num_tokens, num_cols};      \
    const LocalRows<TT> act_rows{(TT*)act_grad, row_id_map, num_tokens, num_cols};                  \
    if (vec)                                                                                        \
      unpermute_bwd_kernel<TT, PP, KM, true><<<grid, kRowWarps * 32, 0, s>>>(                        \
          (const TT*)grad_out, in_rows, act_rows, (const PP*)prob, (PP*)prob_grad, num_tokens,      \
          topk, num_cols);                                                                          \
    else                                                                                            \
      unpermute_bwd_kernel<TT, PP, KM, false><<<grid, kRowWarps * 32, 0, s>>>(                       \
          (const TT*)grad_out, in_rows, act_rows, (const PP*)prob, (PP*)prob_grad, num_tokens,      \
          topk, num_cols);                                                                          \
  }
#define MOE_UB_K(TT, PP)                                                                             \
  if (topk <= 2) { MOE_UB(TT, PP, 2) }                                                              \
  else if (topk <= 4) { MOE_UB(TT, PP, 4) }                                                         \
  else if (topk <= 8) { MOE_UB(TT, PP, 8) }                                                         \
  else if (topk <= 16) { MOE_UB(TT, PP, 16) }                                                       \
  else { MOE_UB(TT, PP, 32) }
#define MOE_UB_P(TT)                                                                                 \
  switch (prob_dtype) {                                                                             \
    case MOE_F32: MOE_UB_K(TT, float) break;                                                        \
    case MOE_F16: MOE_UB_K(TT, __half) break;                                                       \
    default: MOE_UB_K(TT, __nv_bfloat16) break;                                                     \
  }
  switch (dtype) {
    case MOE_F32: MOE_UB_P(float) break;
    case MOE_F16: MOE_UB_P(__half) break;
    default: MOE_UB_P(__nv_bfloat16) break;
  }
#undef MOE_UB_P
#undef MOE_UB_K
#undef MOE_UB
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_gmm_fwd(const void* A, const void* B, void* C, const int32_t* offsets, int32_t num_offsets,
                int64_t m_total, int64_t n, int64_t k, int32_t E, int trans_b, int dtype,
                void* stream) {
  int rc = check_gmm_args(A, B, C, offsets, num_offsets, m_total, n, k, E, dtype);
  if (rc) return rc;
  if (E == 0) return MOE_OK;
  // trans_b: B[e] is [N, K] (K-major operand); else [K, N] (MN-major operand).
  return gmm_rows(A, B, C, offsets, num_offsets == E + 1, m_total, n, k, E, !trans_b, dtype,
                  (cudaStream_t)stream);
}

int moe_gmm_fwd_gather(const void* A_src, const int32_t* a_rows, int64_t a_src_rows, const void* B,
                       void* C, const int32_t* offsets, int32_t num_offsets, int64_t m_total,
                       int64_t n, int64_t k, int32_t E, int trans_b, int dtype, void* stream) {
  int rc = check_gmm_args(A_src, B, C, offsets, num_offsets, m_total, n, k, E, dtype);
  if (rc) return rc;
  if (E == 0 || m_total == 0 || n == 0) return MOE_OK;
  const GatherArgs ga{a_rows, a_src_rows};
  return gmm_rows(A_src, B, C, offsets, num_offsets == E + 1, m_total, n, k, E, !trans_b, dtype,
                  (cudaStream_t)stream, nullptr, nullptr, &ga);
}

int moe_gmm_wgrad_gather(const void* A_src, const int32_t* a_rows, int64_t a_src_rows,
                         const void* grad_C, void* grad_B, const int32_t* offsets,
                         int32_t num_offsets, int64_t m_total, int64_t n, int64_t k, int32_t E,
                         int trans_b, int dtype, void* stream) {
  int rc = check_gmm_args(A_src, grad_C, grad_B, offsets, num_offsets, m_total, n, k, E, dtype);
  if (rc) return rc;
  MOE_REQUIRE(trans_b != 0, "gmm_wgrad_gather: supports trans_b (grad_B [E, N, K]) only");
  if (E == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (m_total == 0) {
    MOE_CUDA_CHECK(cudaMemsetAsync(grad_B, 0, (size_t)E * n * k * dtype_size(dtype), s));
    return MOE_OK;
  }
  const GatherArgs ga{a_rows, a_src_rows};
  return gmm_wgrad(grad_C, A_src, grad_B, offsets, num_offsets == E + 1, m_total, n, k, E, dtype, s,
                   &ga);
}

int moe_gmm_dgrad(const void* grad_C, const void* B, void* grad_A, const int32_t* offsets,
                  int32_t num_offsets, int64_t m_total, int64_t n, int64_t k, int32_t E,
                  int trans_b, int dtype, void* stream) {
  int rc = check_gmm_args(grad_C, B, grad_A, offsets, num_offsets, m_total, n, k, E, dtype);
  if (rc) return rc;
  if (E == 0) return MOE_OK;
  // grad_A [M, K] = grad_C [M, N] . B'[e], contraction over N.  With trans_b, B[e] is
  // [N, K]: contraction rows, output columns contiguous -> MN-major operand.  Without,
  // B[e] is [K, N]: contraction contiguous -> K-major operand.
  return gmm_rows(grad_C, B, grad_A, offsets, num_offsets == E + 1, m_total, k, n, E, trans_b != 0,
                  dtype, (cudaStream_t)stream);
}

int moe_gmm_dgrad_dual(const void* grad_C1, const void* B1, const void* grad_C2, const void* B2,
                       void* grad_A, const int32_t* offsets, int32_t num_offsets, int64_t m_total,
                       int64_t n1, int64_t n2, int64_t k, int32_t E, int trans_b, int dtype,
                       void* stream) {
  int rc = check_gmm_args(grad_C1, B1, grad_A, offsets, num_offsets, m_total, n1, k, E, dtype);
  if (rc) return rc;
  rc = check_gmm_args(grad_C2, B2, grad_A, offsets, num_offsets, m_total, n2, k, E, dtype);
  if (rc) return rc;
  if (E == 0 || m_total == 0 || k == 0) return MOE_OK;
  MOE_REQUIRE(dtype != MOE_F32 && n1 > 0 && n2 > 0 && n1 % 8 == 0 && n2 % 8 == 0 && k % 8 == 0 &&
                  E <= gmm::kMaxGroups && aligned16(grad_C1) && aligned16(grad_C2) &&
                  aligned16(B1) && aligned16(B2) && aligned16(grad_A) && m_total < (1ll << 31) &&
                  n1 < (1ll << 31) && n2 < (1ll << 31) && k < (1ll << 31),
              "gmm_dgrad_dual: needs 16-bit operands, 16-byte aligned, n1, n2 and k multiples "
              "of 8 (the tensor-core path); otherwise call moe_gmm_dgrad twice");
  const RowsSeg2 seg2{grad_C2, B2, n2};
  return gmm_rows(grad_C1, B1, grad_A, offsets, num_offsets == E + 1, m_total, k, n1, E,
                  trans_b != 0, dtype, (cudaStream_t)stream, nullptr, &seg2);
}

int moe_gmm_wgrad(const void* A, const void* grad_C, void* grad_B, const int32_t* offsets,
                  int32_t num_offsets, int64_t m_total, int64_t n, int64_t k, int32_t E,
                  int trans_b, int dtype, void* stream) {
  int rc = check_gmm_args(A, grad_C, grad_B, offsets, num_offsets, m_total, n, k, E, dtype);
  if (rc) return rc;
  if (E == 0) return MOE_OK;
  const int plus_one = num_offsets == E + 1;
  cudaStream_t s = (cudaStream_t)stream;
  if (m_total == 0) {
    MOE_CUDA_CHECK(cudaMemsetAsync(grad_B, 0, (size_t)E * n * k * dtype_size(dtype), s));
    return MOE_OK;
  }
  // trans_b: grad_B[e] [N, K] = grad_C_e^T A_e;  else grad_B[e] [K, N] = A_e^T grad_C_e.
  if (trans_b) return gmm_wgrad(grad_C, A, grad_B, offsets, plus_one, m_total, n, k, E, dtype, s);
  return gmm_wgrad(A, grad_C, grad_B, offsets, plus_one, m_total, k, n, E, dtype, s);
}

}  // extern "C"

static int gate_up_impl(const void* A, const void* B_gate, const void* B_up, void* gate, void* up,
                        void* h, const int32_t* offsets, int32_t num_offsets, int64_t m_total,
                        int64_t n, int64_t k, int32_t E, int trans_b, int dtype, void* stream,
                        const GatherArgs* ga) {
  int rc = check_gmm_args(A, B_gate, gate, offsets, num_offsets, m_total, n, k, E, dtype);
  if (rc) return rc;
  MOE_REQUIRE((B_up && up && h) || m_total == 0 || E == 0, "gmm_gate_up: NULL operand");
  if (E == 0 || m_total == 0 || n == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int plus_one = num_offsets == E + 1;
  const bool tc = dtype != MOE_F32 && k % 8 == 0 && n % 8 == 0 && k > 0 && E <= gmm::kMaxGroups &&
                  aligned16(A) && aligned16(B_gate) && aligned16(B_up) && aligned16(gate) &&
                  aligned16(up) && aligned16(h) && m_total < (1ll << 31) && n < (1ll << 31) &&
                  k < (1ll << 31);
  if (ga) {
    MOE_REQUIRE(tc && ga->rows != nullptr && ga->src_rows > 0 && ga->src_rows < (1ll << 31),
                "gmm_gate_up gather: needs the tensor-core path (16-bit, aligned, sizes multiples "
                "of 8)");
  }
  if (!tc) {
    // Same results from the separate kernels: two grouped GEMMs, then the SwiGLU pass.
    rc = gmm_rows(A, B_gate, gate, offsets, plus_one, m_total, n, k, E, !trans_b, dtype, s);
    if (rc) return rc;
    rc = gmm_rows(A, B_up, up, offsets, plus_one, m_total, n, k, E, !trans_b, dtype, s);
    if (rc) return rc;
    return moe_swiglu_fwd(gate, up, h, m_total * n, dtype, stream);
  }
  CUtensorMap maps[6];  // A, B_gate, h, B_up, gate, up
  {
    const uint64_t dims[2] = {(uint64_t)k, (uint64_t)(ga ? ga->src_rows : m_total)};
    const uint32_t box[2] = {(uint32_t)gmm::BK, ga ? 1u : 64u};
    if ((rc = make_map(&maps[0], A, dtype, 2, dims, box))) return rc;
  }
  for (int i = 0; i < 2; ++i) {
    const void* B = i == 0 ? B_gate : B_up;
    CUtensorMap* m = i == 0 ? &maps[1] : &maps[3];
    if (trans_b) {  // [E, n, k]: K-major, 128 weight rows per box
      const uint64_t dims[3] = {(uint64_t)k, (uint64_t)n, (uint64_t)E};
      const uint32_t box[3] = {(uint32_t)gmm::BK, (uint32_t)(gmm::BN / 2), 1};
      if ((rc = make_map(m, B, dtype, 3, dims, box))) return rc;
    } else {  // [E, k, n]: MN-major, 64-column boxes
      const uint64_t dims[3] = {(uint64_t)n, (uint64_t)k, (uint64_t)E};
      const uint32_t box[3] = {64, (uint32_t)gmm::BK, 1};
      if ((rc = make_map(m, B, dtype, 3, dims, box))) return rc;
    }
  }
  void* outs[3] = {h, gate, up};
  const int out_slot[3] = {2, 4, 5};
  for (int i = 0; i < 3; ++i) {
    const uint64_t dims[2] = {(uint64_t)n, (uint64_t)m_total};
    const uint32_t box[2] = {32, 32};
    if ((rc = make_map(&maps[out_slot[i]], outs[i], dtype, 2, dims, box, CU_TENSOR_MAP_SWIZZLE_64B)))
      return rc;
  }
  gmm::Params p = {};
  p.offsets = offsets;
  p.offsets_plus_one = plus_one;
  p.num_groups = E;
  p.m_total = m_total;
  p.n_out = (int)n;
  p.k_red = (int)k;
  p.out = h;
  p.out_gate = gate;
  p.out_up = up;
  if (ga) {
    p.gather_rows = ga->rows;
    p.gather_src_rows = (int)ga->src_rows;
  }
  const CUtensorMap* extra = &maps[3];
  if (dtype == MOE_BF16)
    return trans_b ? launch_sm100<gmm::kModeGateUp, 1, 1, false, false, __nv_bfloat16>(
                         maps[0], maps[1], maps[2], p, s, extra)
                   : launch_sm100<gmm::kModeGateUp, 1, 1, false, true, __nv_bfloat16>(
                         maps[0], maps[1], maps[2], p, s, extra);
  return trans_b ? launch_sm100<gmm::kModeGateUp, 1, 0, false, false, __half>(maps[0], maps[1],
                                                                             maps[2], p, s, extra)
                 : launch_sm100<gmm::kModeGateUp, 1, 0, false, true, __half>(maps[0], maps[1],
                                                                            maps[2], p, s, extra);
}

extern "C" {

int moe_gmm_gate_up_fwd(const void* A, const void* B_gate, const void* B_up, void* gate,
                        void* up, void* h, const int32_t* offsets, int32_t num_offsets,
                        int64_t m_total, int64_t n, int64_t k, int32_t E, int trans_b, int dtype,
                        void* stream) {
  return gate_up_impl(A, B_gate, B_up, gate, up, h, offsets, num_offsets, m_total, n, k, E, trans_b,
                      dtype, stream, nullptr);
}

int moe_gmm_gate_up_fwd_gather(const void* A_src, const int32_t* a_rows, int64_t a_src_rows,
                               const void* B_gate, const void* B_up, void* gate, void* up, void* h,
                               const int32_t* offsets, int32_t num_offsets, int64_t m_total,
                               int64_t n, int64_t k, int32_t E, int trans_b, int dtype,
                               void* stream) {
  const GatherArgs ga{a_rows, a_src_rows};
  return gate_up_impl(A_src, B_gate, B_up, gate, up, h, offsets, num_offsets, m_total, n, k, E,
                      trans_b, dtype, stream, &ga);
}

int moe_gmm_dgrad_swiglu_bwd(const void* grad_C, const void* B, const void* gate, const void* up,
                             void* grad_gate, void* grad_up, const int32_t* offsets,
                             int32_t num_offsets, int64_t m_total, int64_t n, int64_t k,
                             int32_t E, int trans_b, int dtype, void* stream) {
  int rc = check_gmm_args(grad_C, B, grad_gate, offsets, num_offsets, m_total, n, k, E, dtype);
  if (rc) return rc;
  MOE_REQUIRE((gate && up && grad_up) || m_total == 0 || E == 0, "gmm_dgrad_swiglu_bwd: NULL operand");
  MOE_REQUIRE(aligned16(gate) && aligned16(up) && aligned16(grad_gate) && aligned16(grad_up),
              "gmm_dgrad_swiglu_bwd: gate, up and the gradients must be 16-byte aligned");
  if (E == 0) return MOE_OK;
  const SwiGLUBwdArgs sw = {gate, up, grad_up};
  // As moe_gmm_dgrad: the product is [M, k] = grad_C [M, n] . B'[e].
  return gmm_rows(grad_C, B, grad_gate, offsets, num_offsets == E + 1, m_total, k, n, E,
                  trans_b != 0, dtype, (cudaStream_t)stream, &sw);
}

// ---------------------------------------------------------------- bounded-wait self-test
// One thread waits, with the same bounded wait the GEMM pipeline uses, on an mbarrier that
// nothing arrives at.  The wait gives up after timeout_ns and records device error 1; the
// kernel then returns normally, so the context stays usable.
__global__ void bounded_wait_selftest_kernel(uint64_t timeout_ns, int* result) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_u32(&bar), 1);
    ptx::fence_barrier_init();
    abort_flag = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = ptx::wait_bounded(ptx::smem_u32(&bar), 0, &abort_flag, timeout_ns);
    if (!ok) raise_device_error(1);
    *result = ok ? 1 : 0;
  }
}

// ---------------------------------------------------------------- permute without allocation
// For callers that cannot allocate device memory at call time: code running inside a
// captured stream or a custom allocator's own callbacks, runtimes that pre-plan every
// buffer, or hosts whose only device memory comes from a fixed arena.  The per-tile
// expert counts that moe_permute keeps in caller-provided workspace live instead in this
// file-scope array, which every GPU that loads the library holds until the process exits.
static constexpr size_t kNoAllocScratchInts = 262144;  // 1 MiB: num_tiles * E counts
// moe_permute asks for 16 bytes of workspace beyond the counts, so the array carries them
// too: a request of exactly kNoAllocScratchInts counts must still be accepted.
static constexpr size_t kNoAllocPadInts = 4;
static __device__ __align__(256) int32_t g_permute_scratch[kNoAllocScratchInts + kNoAllocPadInts];
static int32_t* g_permute_scratch_ptr[64] = {nullptr};  // device address, per device

size_t moe_permute_noalloc_max_slots(int32_t E) {
  if (E <= 0) return 0;
  return (kNoAllocScratchInts / (size_t)E) * (size_t)kPermTile;
}

int moe_permute_noalloc(const void* input, int dtype, const int32_t* indices, int64_t num_tokens,
                        int32_t topk, int64_t num_cols, int32_t E, int64_t num_out,
                        void* permuted, int32_t* row_id_map, int32_t* offsets, void* stream) {
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && E > 0,
              "permute_noalloc: bad sizes T=%lld K=%d E=%d", (long long)num_tokens, topk, E);
  const int64_t num_slots = num_tokens * topk;
  const size_t need = (size_t)permute_num_tiles(num_slots) * (size_t)E;
  if (need > kNoAllocScratchInts)
    return set_error(MOE_ERR_INVALID_ARG,
                     "permute_noalloc: T*K=%lld with E=%d needs %zu scratch counts, the fixed "
                     "scratch holds %zu (at most %zu slots for this E); use moe_permute",
                     (long long)num_slots, E, need, kNoAllocScratchInts,
                     moe_permute_noalloc_max_slots(E));
  const int dev = current_device();
  MOE_REQUIRE(dev >= 0 && dev < 64, "permute_noalloc: device %d out of range", dev);
  if (g_permute_scratch_ptr[dev] == nullptr) {
    // One-time set-up on this device (the device is current): the host-side symbol is not
    // a device address, so look the array's device address up.
    void* ptr = nullptr;
    MOE_CUDA_CHECK(cudaGetSymbolAddress(&ptr, g_permute_scratch));
    g_permute_scratch_ptr[dev] = static_cast<int32_t*>(ptr);
  }
  // Every count the kernels read is written first by the histogram kernel of this call,
  // so the array needs no clearing; calls that overlap on the GPU share it and race.
  return moe_permute(input, dtype, indices, num_tokens, topk, num_cols, E, num_out, permuted,
                     row_id_map, offsets, g_permute_scratch_ptr[dev],
                     (kNoAllocScratchInts + kNoAllocPadInts) * sizeof(int32_t), stream);
}

// ---------------------------------------------------------------- expert parallelism over peer memory
int moe_ipc_malloc(size_t bytes, void** ptr, void* handle) {
  MOE_REQUIRE(ptr != nullptr && handle != nullptr && bytes > 0, "ipc_malloc: bad arguments");
  MOE_CUDA_CHECK(cudaMalloc(ptr, bytes));
  const cudaError_t e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return set_error(MOE_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  return MOE_OK;
}

int moe_ipc_open(const void* handle, void** ptr) {
  MOE_REQUIRE(ptr != nullptr && handle != nullptr, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  MOE_CUDA_CHECK(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MOE_OK;
}

int moe_ipc_close(void* ptr) {
  MOE_CUDA_CHECK(cudaIpcCloseMemHandle(ptr));
  return MOE_OK;
}

int moe_ipc_free(void* ptr) {
  MOE_CUDA_CHECK(cudaFree(ptr));
  return MOE_OK;
}

int moe_ep_slot_map(const int32_t* indices, const int32_t* row_id_map, const int32_t* delta,
                    int64_t num_tokens, int32_t topk, int32_t E, int32_t experts_per_rank,
                    int32_t world, int64_t capacity, int32_t* ranks, int32_t* rows, void* stream) {
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && topk <= 32 && E > 0 && experts_per_rank > 0 &&
                  world > 0 && E == experts_per_rank * world && capacity >= 0 &&
                  capacity < (1ll << 31),
              "ep_slot_map: bad sizes T=%lld K=%d E=%d El=%d W=%d", (long long)num_tokens, topk,
              E, experts_per_rank, world);
  const int64_t n = num_tokens * topk;
  if (n == 0) return MOE_OK;
  const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms(current_device()) * 8);
  ep_slot_map_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(indices, row_id_map, delta, num_tokens,
                                                             topk, E, experts_per_rank, world,
                                                             capacity, ranks, rows);
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_ep_dispatch(const void* input, int dtype, void* const* bases, const int32_t* ranks,
                    const int32_t* rows, int64_t num_tokens, int32_t topk, int64_t num_cols,
                    const int32_t* status, void* stream) {
  MOE_REQUIRE(dtype_ok(dtype), "ep_dispatch: bad dtype %d", dtype);
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && topk <= 32 && num_cols >= 0, "ep_dispatch: bad sizes");
  MOE_REQUIRE(aligned16(input), "ep_dispatch: input must be 16-byte aligned");
  if (num_tokens == 0 || num_cols == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  // Receive buffers are 256-byte aligned allocations; rows are 16-byte multiples or not,
  // the same for every rank.
  const bool vec = (num_cols * dtype_size(dtype)) % 16 == 0;
  const dim3 grid((unsigned)((num_tokens + kRowWarps - 1) / kRowWarps));
#define MOE_EPD(TT)                                                                                  \
  {                                                                                                 \
    const PeerRows<TT> r{(TT* const*)bases, ranks, rows, num_tokens, num_cols, status};              \
    if (vec)                                                                                        \
      permute_copy_kernel<TT, true><<<grid, kRowWarps * 32, 0, s>>>((const TT*)input, r,             \
                                                                    num_tokens, topk, num_cols);   \
    else                                                                                            \
      permute_copy_kernel<TT, false><<<grid, kRowWarps * 32, 0, s>>>((const TT*)input, r,            \
                                                                     num_tokens, topk, num_cols);  \
  }
  switch (dtype) {
    case MOE_F32: MOE_EPD(float) break;
    case MOE_F16: MOE_EPD(__half) break;
    default: MOE_EPD(__nv_bfloat16) break;
  }
#undef MOE_EPD
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_ep_combine(const void* const* bases, int dtype, const int32_t* ranks, const int32_t* rows,
                   const void* prob, int prob_dtype, int64_t num_tokens, int32_t topk,
                   int64_t num_cols, void* out, const int32_t* status, void* stream) {
  MOE_REQUIRE(dtype_ok(dtype) && (prob == nullptr || dtype_ok(prob_dtype)),
              "ep_combine: bad dtype %d / prob dtype %d", dtype, prob_dtype);
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && topk <= 32 && num_cols >= 0, "ep_combine: bad sizes");
  MOE_REQUIRE(aligned16(out), "ep_combine: out must be 16-byte aligned");
  if (num_tokens == 0 || num_cols == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const bool vec = (num_cols * dtype_size(dtype)) % 16 == 0;
  const dim3 grid((unsigned)((num_tokens + kRowWarps - 1) / kRowWarps));
  const int pd = prob == nullptr ? MOE_F32 : prob_dtype;
#define MOE_EPC(TT, PP)                                                                              \
  {                                                                                                 \
    const PeerRows<const TT> r{(const TT* const*)bases, ranks, rows, num_tokens, num_cols, status};  \
    MOE_UNP_LAUNCH(TT, PP, r)                                                                       \
  }
#define MOE_EPC_P(TT)                                                                                \
  switch (pd) {                                                                                     \
    case MOE_F32: MOE_EPC(TT, float) break;                                                         \
    case MOE_F16: MOE_EPC(TT, __half) break;                                                        \
    default: MOE_EPC(TT, __nv_bfloat16) break;                                                      \
  }
  switch (dtype) {
    case MOE_F32: MOE_EPC_P(float) break;
    case MOE_F16: MOE_EPC_P(__half) break;
    default: MOE_EPC_P(__nv_bfloat16) break;
  }
#undef MOE_EPC_P
#undef MOE_EPC
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_ep_combine_bwd(const void* grad_out, const void* const* in_bases, void* const* act_bases,
                       int dtype, const int32_t* ranks, const int32_t* rows, const void* prob,
                       int prob_dtype, int64_t num_tokens, int32_t topk, int64_t num_cols,
                       void* prob_grad, const int32_t* status, void* stream) {
  MOE_REQUIRE(dtype_ok(dtype) && dtype_ok(prob_dtype), "ep_combine_bwd: bad dtype");
  MOE_REQUIRE(num_tokens >= 0 && topk > 0 && topk <= 32 && num_cols >= 0, "ep_combine_bwd: bad sizes");
  MOE_REQUIRE(prob != nullptr && prob_grad != nullptr, "ep_combine_bwd: prob / prob_grad is NULL");
  MOE_REQUIRE(aligned16(grad_out), "ep_combine_bwd: grad_out must be 16-byte aligned");
  if (num_tokens == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const bool vec = (num_cols * dtype_size(dtype)) % 16 == 0;
  const dim3 grid((unsigned)((num_tokens + kRowWarps - 1) / kRowWarps));
#define MOE_EPB(TT, PP, KM)                                                                          \
  {                                                                                                 \
    const PeerRows<const TT> ir{(const TT* const*)in_bases, ranks, rows, num_tokens, num_cols,      \
                                status};                                                            \
    const PeerRows<TT> ar{(TT* const*)act_bases, ranks, rows, num_tokens, num_cols, status};        \
    if (vec)                                                                                        \
      unpermute_bwd_kernel<TT, PP, KM, true><<<grid, kRowWarps * 32, 0, s>>>(                        \
          (const TT*)grad_out, ir, ar, (const PP*)prob, (PP*)prob_grad, num_tokens, topk, num_cols);\
    else                                                                                            \
      unpermute_bwd_kernel<TT, PP, KM, false><<<grid, kRowWarps * 32, 0, s>>>(                       \
          (const TT*)grad_out, ir, ar, (const PP*)prob, (PP*)prob_grad, num_tokens, topk, num_cols);\
  }
#define MOE_EPB_K(TT, PP)                                                                            \
  if (topk <= 2) { MOE_EPB(TT, PP, 2) }                                                             \
  else if (topk <= 4) { MOE_EPB(TT, PP, 4) }                                                        \
  else if (topk <= 8) { MOE_EPB(TT, PP, 8) }                                                        \
  else if (topk <= 16) { MOE_EPB(TT, PP, 16) }                                                      \
  else { MOE_EPB(TT, PP, 32) }
#define MOE_EPB_P(TT)                                                                                \
  switch (prob_dtype) {                                                                             \
    case MOE_F32: MOE_EPB_K(TT, float) break;                                                       \
    case MOE_F16: MOE_EPB_K(TT, __half) break;                                                      \
    default: MOE_EPB_K(TT, __nv_bfloat16) break;                                                    \
  }
  switch (dtype) {
    case MOE_F32: MOE_EPB_P(float) break;
    case MOE_F16: MOE_EPB_P(__half) break;
    default: MOE_EPB_P(__nv_bfloat16) break;
  }
#undef MOE_EPB_P
#undef MOE_EPB_K
#undef MOE_EPB
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_add_rows(void* dst, const void* src, const int32_t* n_rows, int64_t max_rows,
                 int64_t num_cols, int dtype, void* stream) {
  MOE_REQUIRE(dtype_ok(dtype) && max_rows >= 0 && num_cols >= 0 && n_rows != nullptr,
              "add_rows: bad arguments");
  if (max_rows == 0 || num_cols == 0) return MOE_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const bool vec = (num_cols * dtype_size(dtype)) % 16 == 0 && aligned16(dst) && aligned16(src);
  const unsigned grid = elementwise_grid(max_rows * num_cols, vec ? 16 / dtype_size(dtype) : 1);
#define MOE_ADD(TT)                                                                                  \
  if (vec) add_rows_kernel<TT, true><<<grid, 256, 0, s>>>((TT*)dst, (const TT*)src, n_rows, max_rows, num_cols); \
  else add_rows_kernel<TT, false><<<grid, 256, 0, s>>>((TT*)dst, (const TT*)src, n_rows, max_rows, num_cols);
  switch (dtype) {
    case MOE_F32: MOE_ADD(float) break;
    case MOE_F16: MOE_ADD(__half) break;
    default: MOE_ADD(__nv_bfloat16) break;
  }
#undef MOE_ADD
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_ep_barrier(int64_t* const* flags, int32_t rank, int32_t world, int64_t* epoch_counter,
                   uint64_t timeout_ns, int32_t* status, void* stream) {
  MOE_REQUIRE(flags != nullptr && epoch_counter != nullptr && world > 0 && world <= 32 &&
                  rank >= 0 && rank < world,
              "ep_barrier: bad arguments rank=%d world=%d", rank, world);
  MOE_REQUIRE(timeout_ns <= 10000000000ull, "ep_barrier: timeout above 10 s");
  ep_barrier_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flags, rank, world, epoch_counter,
                                                         timeout_ns, status);
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_ep_put_counts(const int32_t* counts, int32_t num_experts, int32_t* const* bases,
                      int32_t rank, int32_t world, void* stream) {
  MOE_REQUIRE(counts != nullptr && bases != nullptr && num_experts > 0 && world > 0 &&
                  world <= 32 && rank >= 0 && rank < world,
              "ep_put_counts: bad arguments E=%d rank=%d world=%d", num_experts, rank, world);
  ep_put_counts_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(counts, num_experts, bases, rank, world);
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_write_probe(void* dst, size_t bytes, void* stream) {
  MOE_REQUIRE(aligned16(dst) && bytes % 16 == 0, "write_probe: dst and bytes must be 16-byte multiples");
  if (bytes == 0) return MOE_OK;
  const int64_t n = (int64_t)(bytes / 16);
  write_probe_kernel<<<elementwise_grid(n * 16, 16), 256, 0, (cudaStream_t)stream>>>(
      static_cast<uint4*>(dst), n);
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

int moe_selftest_bounded_wait(uint64_t timeout_ns, int32_t* result, void* stream) {
  MOE_REQUIRE(result != nullptr, "selftest: result is NULL");
  MOE_REQUIRE(timeout_ns <= 10000000000ull, "selftest: timeout above 10 s");
  bounded_wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(timeout_ns, result);
  MOE_LAUNCH_CHECK();
  return MOE_OK;
}

}  // extern "C"
