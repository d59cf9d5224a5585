// CUDA-core grouped GEMM for the requests the tensor-core kernel does not take:
// fp32 operands (the reference runs fp32 through its non-TMA Triton kernel,
// triton_gmm_ops/grouped_gemm_ops.py:20-69 and :126-165) and 16-bit operands whose rows
// are not 16-byte multiples (TMA cannot address them).  Exact fp32 FMA accumulation.
//
// 64x64 output tile per 256-thread block, 4x4 outputs per thread, contraction staged
// through shared memory 16 deep.  Like the reference, the row-mode grid is sized by the
// whole row count per expert slot and tiles past an expert's end return at once, so no
// host synchronisation is needed.
#pragma once

#include "common.cuh"

namespace moe {
namespace simt {

constexpr int TM = 64, TN = 64, TK = 16;

struct GroupRange {
  int64_t start, rows;
};

__device__ __forceinline__ GroupRange group_range(const int32_t* offsets, int plus_one, int g) {
  GroupRange r;
  if (plus_one) { r.start = offsets[g]; r.rows = (int64_t)offsets[g + 1] - offsets[g]; }
  else { r.start = g > 0 ? offsets[g - 1] : 0; r.rows = (int64_t)offsets[g] - r.start; }
  if (r.rows < 0) r.rows = 0;
  return r;
}

// Row mode: C[start+m, n] = sum_k A[start+m, k] * B(g, n, k),
// B(g, n, k) = b_mn ? B[(g*Kc + k)*Nout + n] : B[(g*Nout + n)*Kc + k].
template <typename T>
__global__ void __launch_bounds__(256)
gmm_rows_simt_kernel(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C,
                     const int32_t* __restrict__ offsets, int plus_one, int64_t Nout, int64_t Kc,
                     int b_mn) {
  const int g = blockIdx.z;
  const GroupRange gr = group_range(offsets, plus_one, g);
  const int64_t m0 = (int64_t)blockIdx.x * TM;
  if (m0 >= gr.rows) return;
  const int64_t n0 = (int64_t)blockIdx.y * TN;
  __shared__ float As[TK][TM + 1];
  __shared__ float Bs[TK][TN + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  const T* Bg = B + (int64_t)g * Nout * Kc;
  for (int64_t k0 = 0; k0 < Kc; k0 += TK) {
    for (int i = threadIdx.x; i < TK * TM; i += 256) {
      const int kk = i % TK, mm = i / TK;
      const int64_t m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < gr.rows && k < Kc) ? to_f32(A[(gr.start + m) * Kc + k]) : 0.f;
    }
    for (int i = threadIdx.x; i < TK * TN; i += 256) {
      int kk, nn;
      if (b_mn) { nn = i % TN; kk = i / TN; } else { kk = i % TK; nn = i / TK; }
      const int64_t n = n0 + nn, k = k0 + kk;
      float v = 0.f;
      if (n < Nout && k < Kc) v = to_f32(b_mn ? Bg[k * Nout + n] : Bg[n * Kc + k]);
      Bs[kk][nn] = v;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { a[i] = As[kk][ty * 4 + i]; b[i] = Bs[kk][tx * 4 + i]; }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= gr.rows) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx * 4 + j;
      if (n < Nout) C[(gr.start + m) * Nout + n] = from_f32<T>(acc[i][j]);
    }
  }
}

// Wgrad mode: Out[g, p, q] = sum_{m in expert g} X[m, p] * Y[m, q]  (zeros for empty g).
template <typename T>
__global__ void __launch_bounds__(256)
gmm_wgrad_simt_kernel(const T* __restrict__ X, const T* __restrict__ Y, T* __restrict__ Out,
                      const int32_t* __restrict__ offsets, int plus_one, int64_t P, int64_t Q) {
  const int g = blockIdx.z;
  const GroupRange gr = group_range(offsets, plus_one, g);
  const int64_t p0 = (int64_t)blockIdx.y * TM, q0 = (int64_t)blockIdx.x * TN;
  __shared__ float Xs[TK][TM + 1];
  __shared__ float Ys[TK][TN + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  for (int64_t r0 = 0; r0 < gr.rows; r0 += TK) {
    for (int i = threadIdx.x; i < TK * TM; i += 256) {
      const int pp = i % TM, rr = i / TM;
      const int64_t r = r0 + rr, pi = p0 + pp;
      Xs[rr][pp] = (r < gr.rows && pi < P) ? to_f32(X[(gr.start + r) * P + pi]) : 0.f;
    }
    for (int i = threadIdx.x; i < TK * TN; i += 256) {
      const int qq = i % TN, rr = i / TN;
      const int64_t r = r0 + rr, qi = q0 + qq;
      Ys[rr][qq] = (r < gr.rows && qi < Q) ? to_f32(Y[(gr.start + r) * Q + qi]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int rr = 0; rr < TK; ++rr) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) { a[i] = Xs[rr][ty * 4 + i]; b[i] = Ys[rr][tx * 4 + i]; }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t pi = p0 + ty * 4 + i;
    if (pi >= P) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t qi = q0 + tx * 4 + j;
      if (qi < Q) Out[((int64_t)g * P + pi) * Q + qi] = from_f32<T>(acc[i][j]);
    }
  }
}

}  // namespace simt
}  // namespace moe
