// Persistent Newton-Schulz kernel: every GEMM of every iteration in one launch.
//
// The reference runs three kernels per iteration (csrc/ns_gemm.cu:54-135,
// two SYRK launches and a cuBLAS GEMM) and names the fusion across them as its
// next step (docs/optimization_report.md:260-261: "multi-step NS pipeline —
// persistent kernel across iterations").  Here one grid of one CTA per SM
// walks the work units of all `steps` iterations in order:
//
//   unit = (iteration, phase, matrix of the batch, output tile)
//   phase 0  A  = X·Xᵀ                     lower-triangle tiles, mirrored store
//   phase 1  B  = offdiag(c·A·A + b·A), d = a + diag(c·A·A + b·A)
//   phase 2  X' = d ⊙ X + B·X              (the last iteration writes the output)
//
// with the same warp roles, shared-memory ring, TMEM double buffer and fused
// epilogues as the per-GEMM kernels (ns_gemm_sm100.cuh).  What replaces the
// kernel boundary is a completion counter per phase in global memory: each
// epilogue warp adds one after its stores are fenced; a unit's loads (and its
// epilogue's reads of A or X) start once the phases it reads are complete.
// The pipeline never drains between phases: tiles of the next phase are
// loaded as soon as the phase they read is complete, while this CTA's last
// epilogue of the previous phase may still be storing, there is no launch,
// grid flush, TMEM allocation or barrier set-up per GEMM, and small matrices
// (a few tiles per phase) stop paying those fixed costs fifteen times.
//
// Units are dealt round-robin (unit u to CTA u mod grid) and every unit waits
// only on phases with smaller unit indices, so the lowest unfinished unit can
// always proceed: with all CTAs resident (one per SM, launched cooperatively)
// the schedule cannot deadlock.  Every wait is bounded like the mbarrier waits
// (error code kErrWaitDep), after which the CTA frees its TMEM and exits.
//
// Phase counters: a ring of kFusedSlots ints, zeroed before the launch.
// Phase q accumulates into slot q % kFusedSlots; with a ring length that is a
// multiple of 3, every phase of a slot has the same number of units U, so
// phase q is complete when its slot holds at least (q / kFusedSlots + 1) * 4U
// (phase q + kFusedSlots starts only after phase q is complete).
#pragma once
#include "ns_gemm_sm100.cuh"

namespace fm {

enum : unsigned { kErrWaitDep = 6 };  // a phase-completion wait ran out

constexpr int kFusedSlots = 6;
constexpr int kEpiWarps = 4;

template <int BN>
struct FusedCfg {
  static constexpr int kTileB = BN * kBK * 2;
  static constexpr int kStageBytes = kTileABytes + kTileB;
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256 + kEpiStageBytes;
  static constexpr int kTmemCols = 2 * BN;
};

struct FusedMaps {
  CUtensorMap xk[2];   // X ping-pong buffers, K-major boxes (64 x 128)
  CUtensorMap xmn[2];  // the same, MN-major boxes (64 columns x 64 rows)
  CUtensorMap a;       // A, K-major boxes (both operands of phase 1)
  CUtensorMap b;       // Boff, K-major boxes (A operand of phase 2)
  // epilogue store maps (32 x 32 boxes, no swizzle)
  CUtensorMap so_a, so_b, so_x[2];
  CUtensorMap so_out;  // last iteration's destination (valid when tma_out_final)
};

struct FusedArgs {
  int M, N;            // matrix rows (m) and columns (n), m <= n
  int batch, steps;
  int t_syrk;          // lower-triangle tiles per matrix (phases 0 and 1)
  int tiles_m3, tiles_n3;
  int units_iter;      // units per iteration
  __nv_bfloat16* X[2];
  long long ldx, xs;   // row and matrix strides of the X buffers
  __nv_bfloat16* A;
  __nv_bfloat16* B;
  long long ldm, ms;
  float* diag;
  long long dsz;
  __nv_bfloat16* out;  // last iteration's destination
  long long out_ld, out_bs;
  int transpose_out;
  int tma_out_final;   // 1: the destination has 16-byte aligned rows (so_out valid)
  int* counters;       // kFusedSlots phase counters, zero at launch
  int* rowdone;        // CTA-pair kernel: 2 x tiles_m3 row-block counters of the
                       // B·X phases (iteration parity), zero at launch
  unsigned* err;
};

template <int BN>
__host__ __device__ inline int fused_syrk_tiles(int m) {
  const int mt = (m + kBM - 1) / kBM;
  int cnt = 0;
  for (int i = 0; i < mt; ++i) cnt += (i * kBM + kBM - 1) / BN + 1;
  return cnt;
}

struct FusedUnit {
  int it, p, ph, b, ti, tj;
};

template <int BN>
__device__ __forceinline__ FusedUnit fused_unit(const FusedArgs& f, int u) {
  FusedUnit w;
  w.it = u / f.units_iter;
  int r = u - w.it * f.units_iter;
  const int n1 = f.batch * f.t_syrk;
  int per;
  if (r < n1) {
    w.p = 0;
    per = f.t_syrk;
  } else if (r < 2 * n1) {
    w.p = 1;
    r -= n1;
    per = f.t_syrk;
  } else {
    w.p = 2;
    r -= 2 * n1;
    per = f.tiles_m3 * f.tiles_n3;
  }
  w.b = r / per;
  int t = r - w.b * per;
  if (w.p == 2) {
    w.tj = t / f.tiles_m3;  // column-block-major, as in the per-GEMM kernel
    w.ti = t - w.tj * f.tiles_m3;
  } else {
    int i = 0;
    for (;; ++i) {
      const int c = (i * kBM + kBM - 1) / BN + 1;
      if (t < c) break;
      t -= c;
    }
    w.ti = i;
    w.tj = t;
  }
  w.ph = w.it * 3 + w.p;
  return w;
}

// Epilogue-warp arrivals that complete phase q.
__device__ __forceinline__ int fused_target(const FusedArgs& f, int q) {
  const int units = (q % 3 == 2) ? f.batch * f.tiles_m3 * f.tiles_n3 : f.batch * f.t_syrk;
  return (q / kFusedSlots + 1) * kEpiWarps * units;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Orders this thread's generic-proxy global accesses with later (or, on the
// writing side, other threads' later) async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bounded wait until phase q is complete.  `done_upto` caches the highest
// phase this thread has already seen complete (phases complete in order).
__device__ __forceinline__ bool fused_wait_phase(const FusedArgs& f, int q, int& done_upto,
                                                 volatile int* abort_flag) {
  if (q < 0 || q <= done_upto) return true;
  const int* c = f.counters + (q % kFusedSlots);
  const int target = fused_target(f, q);
  unsigned long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire_gpu(c) >= target) break;
    if ((it & 63u) == 63u) {
      if (*abort_flag) return false;
      const unsigned long long now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitBudgetNs) {
        atomicCAS(f.err, 0u, kErrWaitDep);
        *abort_flag = 1;
        return false;
      }
    }
    __nanosleep(32);
  }
  done_upto = q;
  return true;
}

// GemmArgs of one unit for the shared epilogue code.
__device__ __forceinline__ GemmArgs fused_gemm_args(const FusedArgs& f, const FusedUnit& w) {
  GemmArgs g{};
  g.M = f.M;
  g.err = f.err;
  const long long bm = static_cast<long long>(w.b) * f.ms;
  g.tma_out = 1;
  if (w.p == 0) {
    g.N = f.M;
    g.out = f.A + bm;
    g.ld_out = f.ldm;
  } else if (w.p == 1) {
    g.N = f.M;
    g.out = f.B + bm;
    g.ld_out = f.ldm;
    g.aux = f.A + bm;
    g.ld_aux = f.ldm;
    g.diag = f.diag + static_cast<long long>(w.b) * f.dsz;
  } else {
    g.N = f.N;
    const bool last = w.it == f.steps - 1;
    if (last) {
      g.out = f.out + static_cast<long long>(w.b) * f.out_bs;
      g.ld_out = f.out_ld;
      g.transpose_out = f.transpose_out;
      g.tma_out = f.tma_out_final;
    } else {
      g.out = f.X[(w.it + 1) & 1] + static_cast<long long>(w.b) * f.xs;
      g.ld_out = f.ldx;
    }
    g.aux = f.X[w.it & 1] + static_cast<long long>(w.b) * f.xs;
    g.ld_aux = f.ldx;
    g.diag = f.diag + static_cast<long long>(w.b) * f.dsz;
  }
  return g;
}

#ifdef FM_TRACE
// Development timeline (built only with -DFM_TRACE): per CTA and unit k < 64,
// [0] producer passed its dependency waits, [1] first stage landed (MMA warp),
// [2] accumulator committed, [3] epilogue warp 2 counted the unit.
__device__ unsigned long long g_fused_trace[160][64][4];
#define FM_FTRACE(k, slot) \
  do { if ((k) < 64) g_fused_trace[blockIdx.x][(k)][(slot)] = globaltimer(); } while (0)
#else
#define FM_FTRACE(k, slot) do { } while (0)
#endif

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    ns_fused_kernel(const __grid_constant__ FusedMaps maps, const FusedArgs f) {
  using C = FusedCfg<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* smemA = smem;
  uint8_t* smemB = smem + C::kStages * kTileABytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty_bar = full_bar + C::kStages;
  uint64_t* accf_bar = empty_bar + C::kStages;
  uint64_t* acce_bar = accf_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
  __nv_bfloat16* sbuf = reinterpret_cast<__nv_bfloat16*>(smem + C::kStages * C::kStageBytes + 256);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total = f.steps * f.units_iter;
  const int kb_n = (f.N + kBK - 1) / kBK;  // phase 0 reduces over n
  const int kb_m = (f.M + kBK - 1) / kBK;  // phases 1 and 2 over m

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&maps.xk[0]);
    tma_prefetch_desc(&maps.xk[1]);
    tma_prefetch_desc(&maps.xmn[0]);
    tma_prefetch_desc(&maps.xmn[1]);
    tma_prefetch_desc(&maps.a);
    tma_prefetch_desc(&maps.b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the normalisation kernel's X0 is complete from here on

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int done_upto = -1;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const FusedUnit w = fused_unit<BN>(f, u);
        // Phases whose outputs this unit's operands are: 0 reads X (phase
        // ph-1, the previous iteration's X'), 1 reads A (ph-1), 2 reads B
        // (ph-1) and X (ph-3).
        if (w.p == 2 && !fused_wait_phase(f, w.ph - 3, done_upto, abort_flag)) break;
        if (!fused_wait_phase(f, w.ph - 1, done_upto, abort_flag)) break;
        FM_FTRACE((u - int(blockIdx.x)) / int(gridDim.x), 0);
        fence_proxy_async_global();
        const CUtensorMap* ma = w.p == 0 ? &maps.xk[w.it & 1] : (w.p == 1 ? &maps.a : &maps.b);
        const CUtensorMap* mb = w.p == 0 ? &maps.xk[w.it & 1]
                                         : (w.p == 1 ? &maps.a : &maps.xmn[w.it & 1]);
        const int nkb = w.p == 0 ? kb_n : kb_m;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, f.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], C::kStageBytes);
          uint8_t* sa = smemA + stage * kTileABytes;
          uint8_t* sb = smemB + stage * C::kTileB;
          tma_load_3d(sa, ma, &full_bar[stage], kb * kBK, w.ti * kBM, w.b);
          if (w.p == 2) {
            // X (K = rows, N = contiguous columns): MN-major boxes of 64 columns
#pragma unroll
            for (int q = 0; q < BN / 64; ++q)
              tma_load_3d(sb + q * (kBK * 64 * 2), mb, &full_bar[stage], w.tj * BN + q * 64,
                          kb * kBK, w.b);
          } else {
#pragma unroll
            for (int q = 0; q < BN / kBM; ++q)
              tma_load_3d(sb + q * kTileABytes, mb, &full_bar[stage], kb * kBK,
                          w.tj * BN + q * kBM, w.b);
          }
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    if (lane == 0) pdl_trigger();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_k = make_idesc_bf16(kBM, BN, 0, 0);
      constexpr uint32_t idesc_mn = make_idesc_bf16(kBM, BN, 0, 1);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const int it = u / f.units_iter;
        const int r = u - it * f.units_iter;
        const int p = r < f.batch * f.t_syrk ? 0 : (r < 2 * f.batch * f.t_syrk ? 1 : 2);
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1, abort_flag, f.err, kErrWaitAccEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int nkb = p == 0 ? kb_n : kb_m;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, f.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (kb == 0) FM_FTRACE((u - int(blockIdx.x)) / int(gridDim.x), 1);
          const uint32_t sa = smem_u32(smemA + stage * kTileABytes);
          const uint32_t sb = smem_u32(smemB + stage * C::kTileB);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = make_sdesc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bdesc = p == 2 ? make_sdesc_sw128(sb + k * 2048, kBK * 64 * 2, 1024)
                                          : make_sdesc_sw128(sb + k * 32, 16, 1024);
            tc_mma_bf16(d_tmem, adesc, bdesc, p == 2 ? idesc_mn : idesc_k,
                        (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(&empty_bar[stage]);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&accf_bar[acc]);
        FM_FTRACE((u - int(blockIdx.x)) / int(gridDim.x), 2);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    __nv_bfloat16* wbuf = sbuf + (warp - 2) * (kEpiWarpBytes / 2);
    int acc = 0;
    uint32_t acc_phase = 0;
    int done_upto = -1;
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      const FusedUnit w = fused_unit<BN>(f, u);
      // The epilogue reads A (phase 1) or X and d (phase 2) with plain loads:
      // acquire the phases that wrote them in this thread too.
      bool ok = true;
      if (lane == 0) {
        if (w.p == 2) ok = fused_wait_phase(f, w.ph - 3, done_upto, abort_flag);
        if (ok && w.p >= 1) ok = fused_wait_phase(f, w.ph - 1, done_upto, abort_flag);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      __syncwarp();
      if (!ok) break;
      const GemmArgs g = fused_gemm_args(f, w);
      const bool out_vec = ((reinterpret_cast<uintptr_t>(g.out) | (g.ld_out * 2)) & 15) == 0;
      const bool aux_vec = ((reinterpret_cast<uintptr_t>(g.aux) | (g.ld_aux * 2)) & 15) == 0;
      const uint32_t tacc = tmem_base + acc * BN;
      const int row0w = w.ti * kBM + q * 32;
      const int col0 = w.tj * BN;
      bool done;
      if (w.p == 0) {
        done = epilogue_tile<kSyrk, false, BN>(g, tacc, q, row0w, col0, lane, out_vec, aux_vec,
                                               &accf_bar[acc], acc_phase, abort_flag, wbuf,
                                               &maps.so_a, w.b);
      } else if (w.p == 1) {
        done = epilogue_tile<kPoly, false, BN>(g, tacc, q, row0w, col0, lane, out_vec, aux_vec,
                                               &accf_bar[acc], acc_phase, abort_flag, wbuf,
                                               &maps.so_b, w.b);
      } else {
        const CUtensorMap* so = w.it == f.steps - 1 ? &maps.so_out : &maps.so_x[(w.it + 1) & 1];
        done = epilogue_tile<kBX, false, BN>(g, tacc, q, row0w, col0, lane, out_vec, aux_vec,
                                             &accf_bar[acc], acc_phase, abort_flag, wbuf, so,
                                             w.b);
      }
      if (!done) break;
      if (lane == 0) mbar_arrive(&acce_bar[acc]);  // TMEM accumulator free again
      // Publish this warp's stores: the TMA stores complete (bulk_wait_all),
      // then visible to generic loads (threadfence) and to other CTAs' TMA
      // loads (proxy fence); then count the warp.
      if (lane == 0) bulk_wait_all();
      __syncwarp();
      fence_proxy_async_global();
      __threadfence();
      __syncwarp();
      if (lane == 0) red_release_gpu_add(f.counters + (w.ph % kFusedSlots), 1);
      if (lane == 0 && warp == 2) FM_FTRACE((u - int(blockIdx.x)) / int(gridDim.x), 3);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  if (warp >= 2) {
    if (lane == 0) bulk_wait_all();  // TMA stores done before the CTA exits
    __syncwarp();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

}  // namespace fm
