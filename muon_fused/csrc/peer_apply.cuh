// Fused all-gather + Muon update over NVLink peer memory.
//
// Replaces, for the sharded FusedMuon step, the pair "NCCL all-gather of the
// bf16 updates into a local receive buffer" + "apply pass reading it back":
// every rank reads each owner's packed updates straight from the owner's
// send buffer (CUDA IPC mapping, plain peer loads over NVLink — no multicast)
// and applies p = round(round(p * decay) + alpha * u) in the same pass.  The
// local receive buffer, its HBM write and its read-back disappear.
//
// Ordering: an owner raises flag[bucket] = step (fm_peer_signal, a release
// store at system scope after the bucket's Newton-Schulz kernels completed in
// stream order); a reader block spins on the owner's flag with acquire loads
// before touching the owner's data.  The spin is bounded: past its budget the
// block records an error code and skips its work, so a missing peer cannot
// hang the GPU.  Owners double-buffer their send buffers by step parity, so
// step s+1 never overwrites what a slower peer may still read of step s.
#pragma once
#include <cuda_bf16.h>
#include <cstdint>

#include "../../include/fused_muon.h"
#include "fm_ptx.cuh"
#include "muon_elementwise.cuh"

namespace fm {

enum : unsigned { kErrPeerFlag = 5 };  // a peer's bucket flag never arrived

// Budget of one flag wait: a peer's bucket can lag this rank by a whole
// bucket of Newton-Schulz work (tens of ms); ten seconds means "gone".
constexpr unsigned long long kPeerWaitNs = 10000000000ull;

__global__ void peer_signal_kernel(long long* flag, long long value) {
  __threadfence_system();
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(flag), "l"(value) : "memory");
}

__device__ __forceinline__ long long ld_acquire_sys(const long long* p) {
  long long v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <typename T>
__device__ __forceinline__ void apply_range(T* __restrict__ p, const __nv_bfloat16* __restrict__ u,
                                            long long n, float decay, float alpha) {
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

// Persistent: one block per SM walks the entries in order; for each entry the
// block waits (thread 0, bounded) for the owner's flag, then the grid strides
// over the entry's elements.  One 256-thread block per SM always fits beside
// a running GEMM CTA (192 threads, no shared memory needed here), so this
// kernel can run on a side stream concurrently with the Newton-Schulz work
// without ever keeping it off the SMs.
__global__ void __launch_bounds__(256) peer_gather_apply_kernel(
    const fm_apply_entry* __restrict__ entries, int nentries,
    const __nv_bfloat16* const* __restrict__ peer_src, long long src_shift,
    const long long* const* __restrict__ peer_flags, int flag_index, long long expected,
    unsigned* err_word) {
  __shared__ int ready;
  __shared__ unsigned long long seen;  // owners whose flag this block has observed
  if (threadIdx.x == 0) seen = 0;
  for (int i = 0; i < nentries; ++i) {
    const fm_apply_entry e = entries[i];
    if (threadIdx.x == 0) {
      int ok = (seen >> e.peer) & 1ull;
      if (!ok) {
        const long long* flag = peer_flags[e.peer] + flag_index;
        ok = ld_acquire_sys(flag) >= expected;
        const unsigned long long t0 = globaltimer();
        while (!ok) {
          if (globaltimer() - t0 > kPeerWaitNs) {
            atomicCAS(err_word, 0u, static_cast<unsigned>(kErrPeerFlag));
            break;
          }
          __nanosleep(500);
          ok = ld_acquire_sys(flag) >= expected;
        }
        if (ok) seen |= 1ull << e.peer;
      }
      ready = ok;
    }
    __syncthreads();
    if (ready) {
      const __nv_bfloat16* u = peer_src[e.peer] + src_shift + e.src_offset;
      switch (e.dtype) {
        case FM_DT_F32:
          apply_range(static_cast<float*>(e.param), u, e.numel, e.decay, e.alpha);
          break;
        case FM_DT_BF16:
          apply_range(static_cast<__nv_bfloat16*>(e.param), u, e.numel, e.decay, e.alpha);
          break;
        default:
          apply_range(static_cast<__half*>(e.param), u, e.numel, e.decay, e.alpha);
          break;
      }
    }
    __syncthreads();  // `ready` is rewritten for the next entry
  }
}

}  // namespace fm
