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
constexpr int kFlatUnroll = 8;  // 16-byte loads in flight per thread on the flat path

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

// Per-thread walk over a block's (row, chunk) pairs.  Thread t visits the
// linear indices t + u*blockDim.x + j*kUnroll*blockDim.x (u < kUnroll) of the
// block's row-major chunk range, as a plain linear loop would; the row/chunk
// split of each index is advanced by a precomputed step instead of a 64-bit
// divide per chunk (which made these kernels ALU-bound).
struct ChunkWalk {
  long long r[kUnroll];
  int c[kUnroll];
  int chunks, step_r, step_c;
  __device__ __forceinline__ void init(long long r0, long long nchunks) {
    chunks = static_cast<int>(nchunks);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = static_cast<int>(threadIdx.x + u * blockDim.x);
      r[u] = r0 + i / chunks;
      c[u] = i % chunks;
    }
    const int step = kUnroll * static_cast<int>(blockDim.x);
    step_r = step / chunks;
    step_c = step % chunks;
  }
  __device__ __forceinline__ void advance() {
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      c[u] += step_c;
      r[u] += step_r;
      if (c[u] >= chunks) {
        c[u] -= chunks;
        ++r[u];
      }
    }
  }
};

// bf16(fl32(x / den)) from rcp = fl32(1 / den) without a full division per
// element.  q = fl32(x * rcp) is within 3 fp32 ulps of fl32(x / den) (two
// roundings of at most half an ulp each, plus the quotient's own rounding),
// i.e. within 6 steps of the bit pattern even across a binade edge; both round
// to the same bf16 unless a bf16 rounding midpoint (low 16 bits == 0x8000)
// lies between them.  So q is used unless its low half is within 16 patterns
// of 0x8000, where the exact division decides (Ziv's strategy: a cheap
// approximation, a rounding test, an exact fallback for the rare hard case).
// Also exact for zeros, infinities, NaNs and subnormal quotients.
__device__ __forceinline__ bool near_bf16_midpoint(float q) {
  return (((__float_as_uint(q) & 0xFFFFu) - 0x7FF0u) & 0xFFFFu) <= 32u;
}

// The rule above over an 8-element chunk.  The exact division runs in a
// warp-uniform branch taken only when some lane of the warp has a hard case
// (a ternary select let the compiler compute the division for every element).
__device__ __forceinline__ void div8_for_bf16(float (&x)[8], float den, float rcp) {
  float q[8];
  bool hard = false;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    q[k] = x[k] * rcp;
    hard |= near_bf16_midpoint(q[k]);
  }
  if (__any_sync(__activemask(), hard)) {
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (near_bf16_midpoint(q[k])) q[k] = __fdiv_rn(x[k], den);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) x[k] = q[k];
}

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

// A bf16 matrix stored as one dense run of 16-byte chunks (row stride ==
// cols, cols a multiple of 8, 16-byte aligned): the prep kernels then walk a
// flat chunk array.  Block b of the grid owns chunks [lo, hi) of it.
__device__ __forceinline__ bool flat_ok(const void* p, int dtype, long long cols, long long ld) {
  return bf16_vec_ok(p, dtype, ld) && ld == cols && (cols & 7) == 0;
}

__device__ __forceinline__ void flat_range(long long total, long long& lo, long long& hi) {
  const long long per = (total + gridDim.x - 1) / gridDim.x;
  lo = min(total, per * blockIdx.x);
  hi = min(total, lo + per);
}

// partials[blockIdx.x] = the block's sum of `acc` (warps in a fixed order).
__device__ __forceinline__ void block_sum_store(float acc, float* partials) {
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

// partials[b][blockIdx.x] = sum over this block's part of bf16(G_b)^2 (fp32);
// blockIdx.y = b, the matrix of the batch (element stride bs_g).
__global__ void __launch_bounds__(kPrepThreads, 4) sumsq_kernel(const void* __restrict__ G0, int dtype,
                                                             long long rows, long long cols,
                                                             long long ldg, long long bs_g,
                                                             float* partials) {
  pdl_wait();
  const void* G = batch_ptr(G0, dtype, bs_g, blockIdx.y);
  partials += static_cast<long long>(blockIdx.y) * kMaxPartials;
  const ChunkGrid g{rows, cols, ldg, (cols + 7) / 8};
  const bool vec = bf16_vec_ok(G, dtype, ldg);
  float acc = 0.f;
  if (flat_ok(G, dtype, cols, ldg)) {
    // Raw 16-byte loads first (4 registers each), so that kFlatUnroll of them
    // are in flight per thread at the register budget of four blocks per SM.
    const uint4* src = static_cast<const uint4*>(G);
    long long lo, hi;
    flat_range(rows * g.chunks, lo, hi);
    for (long long l0 = lo + threadIdx.x; l0 < hi; l0 += kFlatUnroll * blockDim.x) {
      uint4 raw[kFlatUnroll];
#pragma unroll
      for (int u = 0; u < kFlatUnroll; ++u) {
        const long long l = l0 + u * static_cast<long long>(blockDim.x);
        raw[u] = l < hi ? __ldg(src + l) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kFlatUnroll; ++u) {
        float x[8];
        unpack8(raw[u], x);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = fmaf(x[k], x[k], acc);
      }
    }
    block_sum_store(acc, partials);
    pdl_trigger();
    return;
  }
  long long r0, r1;
  g.block_rows(r0, r1);
  ChunkWalk w;
  w.init(r0, g.chunks);
  while (w.r[0] < r1) {
    float x[kUnroll][8];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (w.r[u] < r1) {
        load_chunk(G, dtype, g, vec, w.r[u], w.c[u], x[u]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) x[u][k] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
#pragma unroll
      for (int k = 0; k < 8; ++k) acc = fmaf(x[u][k], x[u][k], acc);
    w.advance();
  }
  block_sum_store(acc, partials);
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
__global__ void __launch_bounds__(kPrepThreads, 4) scale_kernel(const void* __restrict__ G0, int dtype,
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
  const float rcp = 1.f / den;
  if (vout && ldx == cols && flat_ok(G, dtype, cols, ldg)) {
    const uint4* src = static_cast<const uint4*>(G);
    uint4* dst = reinterpret_cast<uint4*>(X);
    long long lo, hi;
    flat_range(rows * g.chunks, lo, hi);
    for (long long l0 = lo + threadIdx.x; l0 < hi; l0 += kFlatUnroll * blockDim.x) {
      uint4 raw[kFlatUnroll];
#pragma unroll
      for (int u = 0; u < kFlatUnroll; ++u) {
        const long long l = l0 + u * static_cast<long long>(blockDim.x);
        if (l < hi) raw[u] = __ldg(src + l);
      }
#pragma unroll
      for (int u = 0; u < kFlatUnroll; ++u) {
        const long long l = l0 + u * static_cast<long long>(blockDim.x);
        if (l >= hi) continue;
        float x[8];
        unpack8(raw[u], x);
        div8_for_bf16(x, den, rcp);
        dst[l] = pack8(x);
      }
    }
    pdl_trigger();
    return;
  }
  long long r0, r1;
  g.block_rows(r0, r1);
  ChunkWalk w;
  w.init(r0, g.chunks);
  for (; w.r[0] < r1; w.advance()) {
    float x[kUnroll][8];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (w.r[u] < r1) load_chunk(G, dtype, g, vin, w.r[u], w.c[u], x[u]);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (w.r[u] >= r1) continue;
      const long long r = w.r[u], c = w.c[u];
      div8_for_bf16(x[u], den, rcp);
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
// Tiles of kTR rows x kTC columns of G go through shared memory so both the
// read (rows of G) and the write (rows of X = columns of G) coalesce; each
// thread has kPer 16-byte chunks in flight.  The tile's row pitch of kTC + 2
// elements keeps the column-wise gathers of the store phase to at most
// two-way bank conflicts and the row-wise writes of the load phase
// conflict-free.
constexpr int kTR = 64;    // rows of G per tile (= columns of the X tile)
constexpr int kTC = 128;   // columns of G per tile (= rows of the X tile)
constexpr int kTPitchT = kTC + 2;
__global__ void __launch_bounds__(kPrepThreads) scale_transpose_kernel(
    const void* __restrict__ G0, int dtype, long long rows, long long cols, long long ldg,
    long long bs_g, const float* partials, int nparts, __nv_bfloat16* X, long long ldx,
    long long xs) {
  pdl_wait();
  const void* G = batch_ptr(G0, dtype, bs_g, blockIdx.z);
  partials += static_cast<long long>(blockIdx.z) * kMaxPartials;
  X += static_cast<long long>(blockIdx.z) * xs;
  __shared__ float s_den;
  __shared__ __nv_bfloat16 tile[kTR][kTPitchT];
  const ChunkGrid g{rows, cols, ldg, (cols + 7) / 8};
  const bool vin = bf16_vec_ok(G, dtype, ldg);
  const bool vout = ((reinterpret_cast<uintptr_t>(X) | static_cast<uintptr_t>(ldx * 2)) & 15) == 0;
  const long long r0 = static_cast<long long>(blockIdx.y) * kTR;
  const long long c0 = static_cast<long long>(blockIdx.x) * kTC;
  constexpr int kPer = kTR * (kTC / 8) / kPrepThreads;  // chunks per thread (4)
  // load: kTR rows x kTC/8 chunks, issued before the norm is reduced
  float x[kPer][8];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = threadIdx.x + j * kPrepThreads;
    const long long r = r0 + i / (kTC / 8), cc = c0 / 8 + i % (kTC / 8);
    if (r < rows && cc * 8 < cols) {
      load_chunk(G, dtype, g, vin, r, cc, x[j]);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) x[j][k] = 0.f;
    }
  }
  const float den = nparts > 0 ? norm_denominator(partials, nparts, &s_den) : 1.f;
  const float rcp = 1.f / den;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = threadIdx.x + j * kPrepThreads;
    const int tr = i / (kTC / 8), tc = i % (kTC / 8);
    div8_for_bf16(x[j], den, rcp);
#pragma unroll
    for (int k = 0; k < 8; ++k) tile[tr][tc * 8 + k] = __float2bfloat16_rn(x[j][k]);
  }
  __syncthreads();
  // store: output rows c0 .. c0+kTC-1, each kTR/8 chunks along r
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = threadIdx.x + j * kPrepThreads;
    const int orow = i / (kTR / 8), oc = i % (kTR / 8);
    const long long c = c0 + orow;    // output row
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
