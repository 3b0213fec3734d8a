// Fused elementwise kernels of the Muon update (reference
// muon_fused/optimizer.py:139-163), one HBM pass each instead of the
// reference's 3 + 2 ATen passes:
//
//   momentum:  buf = bf(bf(buf * mu) + g);  dir = bf(g + mu * buf)  (nesterov)
//              (optimizer.py:144-147: buf.mul_(mu).add_(g); g.add(buf, alpha=mu))
//   apply:     p = bf(bf(p * (1 - lr*wd)) + alpha * u),  alpha = -lr'
//              (optimizer.py:161-163: p.mul_(1 - lr*wd); p.add_(u, alpha=-lr'))
//
// bf(.) is rounding to the tensor's dtype after every torch op, reproduced
// exactly (no contraction of the separate mul and add; the alpha-scaled add
// is one fused multiply-add, as torch's add kernel computes it), so results
// are bit-identical to the reference's torch ops on the same device.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace fm {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

constexpr int kEwThreads = 256;

// 8 consecutive elements as floats; 16-byte vector accesses when `vec`
// (the pointer is 16-byte aligned), element accesses otherwise.
template <typename T>
__device__ __forceinline__ void load8(const T* p, bool vec, float (&x)[8]) {
  if (vec) {
    if constexpr (sizeof(T) == 4) {
      const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
      const float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
      x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(p));
      const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) x[k] = to_f(h[k]);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = to_f(p[k]);
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, bool vec, const float (&x)[8]) {
  if (vec) {
    if constexpr (sizeof(T) == 4) {
      __stcs(reinterpret_cast<float4*>(p), make_float4(x[0], x[1], x[2], x[3]));
      __stcs(reinterpret_cast<float4*>(p) + 1, make_float4(x[4], x[5], x[6], x[7]));
    } else {
      uint4 u;
      T* h = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) h[k] = from_f<T>(x[k]);
      __stcs(reinterpret_cast<uint4*>(p), u);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) p[k] = from_f<T>(x[k]);
  }
}

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

// One element of the momentum update (exact torch rounding, see top).
template <typename T>
__device__ __forceinline__ void momentum1(float& b, float g, float mu, int nesterov, float& d) {
  const float b1 = to_f(from_f<T>(__fmul_rn(b, mu)));
  b = to_f(from_f<T>(__fadd_rn(b1, g)));
  // the direction is rounded to its own dtype first (as torch would), then to bf16
  d = nesterov ? to_f(from_f<T>(fmaf(mu, b, g))) : b;
}

// Momentum update; the direction is written as bf16, the Newton-Schulz input
// type.  Eight elements per thread per iteration, 16-byte accesses when aligned.
template <typename T>
__global__ void __launch_bounds__(kEwThreads) muon_momentum_bf16dir_kernel(
    T* __restrict__ buf, const T* __restrict__ grad, __nv_bfloat16* __restrict__ dir, long long n,
    float mu, int nesterov) {
  const bool vec = aligned16(buf) && aligned16(grad) && aligned16(dir);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long chunks = n / 8;
  for (long long c = tid; c < chunks; c += stride) {
    float b[8], g[8], d[8];
    load8(buf + 8 * c, vec, b);
    load8(grad + 8 * c, vec, g);
#pragma unroll
    for (int k = 0; k < 8; ++k) momentum1<T>(b[k], g[k], mu, nesterov, d[k]);
    store8(buf + 8 * c, vec, b);
    store8(dir + 8 * c, vec, d);
  }
  for (long long i = chunks * 8 + tid; i < n; i += stride) {
    float b = to_f(buf[i]), d;
    momentum1<T>(b, to_f(grad[i]), mu, nesterov, d);
    buf[i] = from_f<T>(b);
    dir[i] = __float2bfloat16_rn(d);
  }
}

template <typename T>
__global__ void __launch_bounds__(kEwThreads) muon_apply_kernel(T* __restrict__ p,
                                                                const __nv_bfloat16* __restrict__ u,
                                                                long long n, float decay,
                                                                float alpha) {
  const bool vec = aligned16(p) && aligned16(u);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long tid = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  const long long chunks = n / 8;
  for (long long c = tid; c < chunks; c += stride) {
    float pv[8], uv[8];
    load8(p + 8 * c, vec, pv);
    load8(u + 8 * c, vec, uv);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      pv[k] = fmaf(alpha, uv[k], to_f(from_f<T>(__fmul_rn(pv[k], decay))));
    store8(p + 8 * c, vec, pv);
  }
  for (long long i = chunks * 8 + tid; i < n; i += stride) {
    const float p1 = to_f(from_f<T>(__fmul_rn(to_f(p[i]), decay)));
    p[i] = from_f<T>(fmaf(alpha, __bfloat162float(u[i]), p1));
  }
}

}  // namespace fm
