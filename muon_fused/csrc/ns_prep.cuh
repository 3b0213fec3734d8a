// Bandwidth kernels around the Newton-Schulz GEMMs: Frobenius norm and the
// fused cast + scale (+ transpose for tall inputs) that produces X0.
//
// Reference behaviour (muon_fused/ns_step.py:40-45, csrc/torch_binding.cu:64-71,91):
//   X = G.bfloat16(); if G.size(0) > G.size(1): X = X.T;  X = X / (||X||_F + 1e-7)
// The reference does this as 3-4 separate ATen passes; here it is two passes:
// one read of G for the sum of squares (per-block partials, no atomics, so the
// norm is bit-reproducible), and one read of G + one write of X0.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace fm {

// Input element codes of the C ABI (fm_dtype in include/fused_muon.h).
enum : int { kDtBF16 = 0, kDtF16 = 1, kDtF32 = 2, kDtF64 = 3 };

constexpr int kPrepThreads = 256;
constexpr int kMaxPartials = 1024;

// Value of G[i] after the reference's cast to bf16, widened to fp32.
__device__ __forceinline__ float load_bf16_rounded(const void* G, int dtype, long long i) {
  switch (dtype) {
    case kDtBF16:
      return __bfloat162float(static_cast<const __nv_bfloat16*>(G)[i]);
    case kDtF16:
      return __bfloat162float(__float2bfloat16_rn(__half2float(static_cast<const __half*>(G)[i])));
    case kDtF32:
      return __bfloat162float(__float2bfloat16_rn(static_cast<const float*>(G)[i]));
    default:
      return __bfloat162float(__double2bfloat16(static_cast<const double*>(G)[i]));
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// partials[blockIdx.x] = sum over this block's rows of bf16(G)^2 (fp32).
// Rows are strided over blocks; columns over threads, 8 at a time when the
// input is bf16 with 16-byte aligned rows.
__global__ void __launch_bounds__(kPrepThreads) sumsq_kernel(const void* __restrict__ G, int dtype,
                                                             long long rows, long long cols,
                                                             long long ldg, float* partials) {
  float acc = 0.f;
  const bool vec = dtype == kDtBF16 && (cols % 8 == 0) && (ldg % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(G) & 15) == 0);
  // Thread t always owns the 8-element chunks t, t + blockDim, ... of a row and
  // accumulates them in element order, whatever the input type, so the norm
  // depends only on the bf16 values.
  const long long chunks = (cols + 7) / 8;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    for (long long c = threadIdx.x; c < chunks; c += blockDim.x) {
      float x[8];
      if (vec) {
        uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(G) + r * ldg) + c);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
          x[2 * k] = f.x;
          x[2 * k + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          x[k] = (c * 8 + k < cols) ? load_bf16_rounded(G, dtype, r * ldg + c * 8 + k) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) acc = fmaf(x[k], x[k], acc);
    }
  }
  __shared__ float red[kPrepThreads / 32];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kPrepThreads / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) partials[blockIdx.x] = v;
  }
}

// Denominator ||G||_F + 1e-7, reduced from the partials in a fixed order.
__device__ __forceinline__ float norm_denominator(const float* partials, int nparts, float* shared_slot) {
  if (threadIdx.x < 32) {
    float v = 0.f;
    for (int i = threadIdx.x; i < nparts; i += 32) v += partials[i];
    v = warp_sum(v);
    if (threadIdx.x == 0) *shared_slot = sqrtf(v) + 1e-7f;
  }
  __syncthreads();
  return *shared_slot;
}

// X[r][c] = bf16(bf16(G[r][c]) / (||G|| + 1e-7)), same layout as G.
// With nparts == 0 no normalisation is applied (plain cast/copy).
__global__ void __launch_bounds__(kPrepThreads) scale_kernel(const void* __restrict__ G, int dtype,
                                                             long long rows, long long cols,
                                                             long long ldg, const float* partials,
                                                             int nparts, __nv_bfloat16* X,
                                                             long long ldx) {
  __shared__ float s_den;
  const float den = nparts > 0 ? norm_denominator(partials, nparts, &s_den) : 1.f;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
      const float x = load_bf16_rounded(G, dtype, r * ldg + c);
      X[r * ldx + c] = __float2bfloat16_rn(x / den);
    }
  }
}

// Transposing variant for tall G (rows > cols): X[c][r] = bf16(bf16(G[r][c]) / den).
// 64x64 tiles through shared memory so both the read and the write coalesce.
constexpr int kTT = 64;
__global__ void __launch_bounds__(kPrepThreads) scale_transpose_kernel(
    const void* __restrict__ G, int dtype, long long rows, long long cols, long long ldg,
    const float* partials, int nparts, __nv_bfloat16* X, long long ldx) {
  __shared__ float s_den;
  __shared__ __nv_bfloat16 tile[kTT][kTT + 2];
  const float den = nparts > 0 ? norm_denominator(partials, nparts, &s_den) : 1.f;
  const long long r0 = static_cast<long long>(blockIdx.y) * kTT;
  const long long c0 = static_cast<long long>(blockIdx.x) * kTT;
  const int tx = threadIdx.x & 63;
  const int ty = threadIdx.x >> 6;  // 0..3
  for (int i = ty; i < kTT; i += kPrepThreads / kTT) {
    const long long r = r0 + i, c = c0 + tx;
    float x = 0.f;
    if (r < rows && c < cols) x = load_bf16_rounded(G, dtype, r * ldg + c) / den;
    tile[i][tx] = __float2bfloat16_rn(x);
  }
  __syncthreads();
  for (int i = ty; i < kTT; i += kPrepThreads / kTT) {
    const long long c = c0 + i, r = r0 + tx;  // output row c, column r
    if (c < cols && r < rows) X[c * ldx + r] = tile[tx][i];
  }
}

}  // namespace fm
