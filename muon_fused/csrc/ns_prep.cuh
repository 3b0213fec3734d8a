// Bandwidth kernels around the Newton-Schulz GEMMs: Frobenius norm and the
// fused cast + scale (+ transpose for tall inputs) that produces X0.
//
// Reference behaviour (muon_fused/ns_step.py:40-45, csrc/torch_binding.cu:64-71,91):
//   X = G.bfloat16(); if G.size(0) > G.size(1): X = X.T;  X = X / (||X||_F + 1e-7)
// The reference does this as 3-4 separate ATen passes; here it is two passes:
// one read of G for the sum of squares (per-block partials, no atomics, so the
// norm is bit-reproducible), and one read of G + one write of X0.
//
// Work unit: an 8-element chunk of a row (16 bytes of bf16).  Each block owns
// a contiguous range of rows and walks its (row, chunk) pairs with four
// chunks in flight per thread; 16-byte loads/stores are used whenever the
// pointer and row stride allow, otherwise element loads with the same
// accumulation order (so the norm depends only on the bf16 values).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "fm_ptx.cuh"

namespace fm {

// Input element codes of the C ABI (FM_DT_* in include/fused_muon.h).
enum : int { kDtBF16 = 0, kDtF16 = 1, kDtF32 = 2, kDtF64 = 3 };

constexpr int kPrepThreads = 256;
constexpr int kMaxPartials = 1024;
constexpr int kUnroll = 4;

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

__device__ __forceinline__ void unpack8(uint4 u, float (&x)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
    x[2 * k] = f.x;
    x[2 * k + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&x)[8]) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * k], x[2 * k + 1]);
    w[k] = *reinterpret_cast<uint32_t*>(&h);
  }
  return u;
}

// Geometry of one prep launch over a rows x cols input with row stride ld.
struct ChunkGrid {
  long long rows, cols, ld;
  long long chunks;  // 8-element chunks per row
  __device__ __forceinline__ void block_rows(long long& r0, long long& r1) const {
    const long long per = (rows + gridDim.x - 1) / gridDim.x;
    r0 = min(rows, per * blockIdx.x);
    r1 = min(rows, r0 + per);
  }
};

// Load chunk (r, c) as bf16-rounded floats (zero beyond cols).
__device__ __forceinline__ void load_chunk(const void* G, int dtype, const ChunkGrid& g, bool vec,
                                           long long r, long long c, float (&x)[8]) {
  const long long base = r * g.ld + c * 8;
  if (vec && c * 8 + 8 <= g.cols) {
    unpack8(__ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(G) + base)), x);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = (c * 8 + k < g.cols) ? load_bf16_rounded(G, dtype, base + k) : 0.f;
  }
}

// Matrix b of a batch: element offset b * bs of an input of the given dtype.
__device__ __forceinline__ const void* batch_ptr(const void* G, int dtype, long long bs, int b) {
  const size_t esz = dtype == kDtF32 ? 4 : dtype == kDtF64 ? 8 : 2;
  return static_cast<const char*>(G) + static_cast<long long>(b) * bs * esz;
}

__device__ __forceinline__ bool bf16_vec_ok(const void* p, int dtype, long long ld) {
  return dtype == kDtBF16 && ((reinterpret_cast<uintptr_t>(p) | static_cast<uintptr_t>(ld * 2)) & 15) == 0;
}

// partials[b][blockIdx.x] = sum over this block's rows of bf16(G_b)^2 (fp32);
// blockIdx.y = b, the matrix of the batch (element stride bs_g).
__global__ void __launch_bounds__(kPrepThreads) sumsq_kernel(const void* __restrict__ G0, int dtype,
                                                             long long rows, long long cols,
                                                             long long ldg, long long bs_g,
                                                             float* partials) {
  pdl_wait();
  const void* G = batch_ptr(G0, dtype, bs_g, blockIdx.y);
  partials += static_cast<long long>(blockIdx.y) * kMaxPartials;
  const ChunkGrid g{rows, cols, ldg, (cols + 7) / 8};
  const bool vec = bf16_vec_ok(G, dtype, ldg);
  long long r0, r1;
  g.block_rows(r0, r1);
  const long long total = (r1 - r0) * g.chunks;
  float acc = 0.f;
  for (long long i0 = threadIdx.x; i0 < total; i0 += kUnroll * blockDim.x) {
    float x[kUnroll][8];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long i = i0 + u * blockDim.x;
      if (i < total) {
        const long long r = r0 + i / g.chunks, c = i % g.chunks;
        load_chunk(G, dtype, g, vec, r, c, x[u]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) x[u][k] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int k = 0; k < 8; ++k) acc = fmaf(x[u][k], x[u][k], acc);
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
  pdl_trigger();
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

// X[r][c] = bf16(bf16(G[r][c]) / (||G|| + 1e-7)), same layout as G;
// blockIdx.y = matrix of the batch (element strides bs_g in, xs out).
// With nparts == 0 no normalisation is applied (plain cast/copy).
__global__ void __launch_bounds__(kPrepThreads) scale_kernel(const void* __restrict__ G0, int dtype,
                                                             long long rows, long long cols,
                                                             long long ldg, long long bs_g,
                                                             const float* partials, int nparts,
                                                             __nv_bfloat16* X, long long ldx,
                                                             long long xs) {
  pdl_wait();
  const void* G = batch_ptr(G0, dtype, bs_g, blockIdx.y);
  if (partials) partials += static_cast<long long>(blockIdx.y) * kMaxPartials;
  X += static_cast<long long>(blockIdx.y) * xs;
  __shared__ float s_den;
  const float den = nparts > 0 ? norm_denominator(partials, nparts, &s_den) : 1.f;
  const ChunkGrid g{rows, cols, ldg, (cols + 7) / 8};
  const bool vin = bf16_vec_ok(G, dtype, ldg);
  const bool vout = ((reinterpret_cast<uintptr_t>(X) | static_cast<uintptr_t>(ldx * 2)) & 15) == 0;
  long long r0, r1;
  g.block_rows(r0, r1);
  const long long total = (r1 - r0) * g.chunks;
  for (long long i0 = threadIdx.x; i0 < total; i0 += kUnroll * blockDim.x) {
    float x[kUnroll][8];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long i = i0 + u * blockDim.x;
      if (i < total) load_chunk(G, dtype, g, vin, r0 + i / g.chunks, i % g.chunks, x[u]);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long i = i0 + u * blockDim.x;
      if (i >= total) continue;
      const long long r = r0 + i / g.chunks, c = i % g.chunks;
#pragma unroll
      for (int k = 0; k < 8; ++k) x[u][k] = x[u][k] / den;
      __nv_bfloat16* dst = X + r * ldx + c * 8;
      if (vout && c * 8 + 8 <= cols) {
        *reinterpret_cast<uint4*>(dst) = pack8(x[u]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (c * 8 + k < cols) dst[k] = __float2bfloat16_rn(x[u][k]);
      }
    }
  }
  pdl_trigger();
}

// Transposing variant for tall G (rows > cols): X[c][r] = bf16(bf16(G[r][c]) / den).
// 64x64 tiles through shared memory so both the read and the write coalesce.
constexpr int kTT = 64;
__global__ void __launch_bounds__(kPrepThreads) scale_transpose_kernel(
    const void* __restrict__ G0, int dtype, long long rows, long long cols, long long ldg,
    long long bs_g, const float* partials, int nparts, __nv_bfloat16* X, long long ldx,
    long long xs) {
  pdl_wait();
  const void* G = batch_ptr(G0, dtype, bs_g, blockIdx.z);
  partials += static_cast<long long>(blockIdx.z) * kMaxPartials;
  X += static_cast<long long>(blockIdx.z) * xs;
  __shared__ float s_den;
  __shared__ __align__(16) __nv_bfloat16 tile[kTT][kTT + 8];
  const float den = nparts > 0 ? norm_denominator(partials, nparts, &s_den) : 1.f;
  const ChunkGrid g{rows, cols, ldg, (cols + 7) / 8};
  const bool vin = bf16_vec_ok(G, dtype, ldg);
  const bool vout = ((reinterpret_cast<uintptr_t>(X) | static_cast<uintptr_t>(ldx * 2)) & 15) == 0;
  const long long r0 = static_cast<long long>(blockIdx.y) * kTT;
  const long long c0 = static_cast<long long>(blockIdx.x) * kTT;
  // load: 64 rows x 8 chunks, two per thread
  for (int i = threadIdx.x; i < kTT * (kTT / 8); i += kPrepThreads) {
    const int tr = i / (kTT / 8), tc = i % (kTT / 8);
    const long long r = r0 + tr, cc = c0 / 8 + tc;
    float x[8];
    if (r < rows) {
      load_chunk(G, dtype, g, vin, r, cc, x);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[tr][tc * 8 + k] = __float2bfloat16_rn(x[k] / den);
  }
  __syncthreads();
  // store: output rows c0.. (64 of them) x 8 chunks along r
  for (int i = threadIdx.x; i < kTT * (kTT / 8); i += kPrepThreads) {
    const int orow = i / (kTT / 8), oc = i % (kTT / 8);
    const long long c = c0 + orow;  // output row
    const long long r = r0 + oc * 8;  // first output column
    if (c >= cols) continue;
    __nv_bfloat16* dst = X + c * ldx + r;
    if (vout && r + 8 <= rows) {
      __align__(16) __nv_bfloat16 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = tile[oc * 8 + k][orow];
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(v);
    } else {
      for (int k = 0; k < 8 && r + k < rows; ++k) dst[k] = tile[oc * 8 + k][orow];
    }
  }
  pdl_trigger();
}

}  // namespace fm
