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

// Momentum update; the direction is written as bf16, the Newton-Schulz input type.
template <typename T>
__global__ void __launch_bounds__(kEwThreads) muon_momentum_bf16dir_kernel(
    T* __restrict__ buf, const T* __restrict__ grad, __nv_bfloat16* __restrict__ dir, long long n,
    float mu, int nesterov) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float g = to_f(grad[i]);
    const float b1 = to_f(from_f<T>(__fmul_rn(to_f(buf[i]), mu)));
    const float b2 = to_f(from_f<T>(__fadd_rn(b1, g)));
    buf[i] = from_f<T>(b2);
    // the direction is rounded to its own dtype first (as torch would), then to bf16
    const float d = nesterov ? to_f(from_f<T>(fmaf(mu, b2, g))) : b2;
    dir[i] = __float2bfloat16_rn(d);
  }
}

template <typename T>
__global__ void __launch_bounds__(kEwThreads) muon_apply_kernel(T* __restrict__ p,
                                                                const __nv_bfloat16* __restrict__ u,
                                                                long long n, float decay,
                                                                float alpha) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float p1 = to_f(from_f<T>(__fmul_rn(to_f(p[i]), decay)));
    p[i] = from_f<T>(fmaf(alpha, __bfloat162float(u[i]), p1));
  }
}

}  // namespace fm
