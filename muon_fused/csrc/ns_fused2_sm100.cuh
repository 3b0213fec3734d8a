// Persistent Newton-Schulz kernel on CTA-pair 256 x 256 tiles, for single
// matrices too large for one wave of 128 x 128 tiles but whose X still sits in
// L2 (e.g. 2560² .. 4096², 4096 x 6144).
//
// It is the CTA-pair GEMM machinery of ns_gemm2_sm100.cuh (2-CTA clusters,
// cta_group::2 MMAs issued by the even CTA, each CTA loading its own halves,
// no multicast) driven by the unit walk and phase counters of
// ns_fused_sm100.cuh, plus one finer dependency that the kernel boundary
// could not express: the next iteration's X·Xᵀ tile (I, J) needs only row
// blocks I and J of X', so it starts as soon as the B·X phase has finished
// those rows.  B·X therefore walks its tiles row-block by row-block, and each
// finished B·X unit also counts into its row block's counter.  The idle CTA
// pairs of B·X's last partial wave and its last epilogues then overlap the
// next iteration's first SYRK tiles.  The other two boundaries stay whole
// phases: A·A needs every row of A, and B·X needs every row of B.
//
// Row counters: 2 x T ints (T = row blocks), iteration parity it & 1; row block
// I of iteration it is done at (it / 2 + 1) x 8 x tiles_n arrivals (eight
// epilogue warps per pair unit).  The slot of iteration it + 2 receives
// arrivals only after every unit of iteration it + 1's X·Xᵀ has passed its
// waits, so the monotonic targets stay exact.  Deadlock freedom as in the
// single-CTA kernel: every wait is on units with smaller indices.
#pragma once
#include "ns_fused_sm100.cuh"
#include "ns_gemm2_sm100.cuh"

namespace fm {

constexpr int kPairEpiWarps = 8;  // 4 epilogue warps in each CTA of the pair

struct PairFusedUnit {
  int it, p, ph, b, ti, tj;
};

__device__ __forceinline__ PairFusedUnit pair_fused_unit(const FusedArgs& f, int u) {
  PairFusedUnit w;
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
  const int t = r - w.b * per;
  if (w.p == 2) {
    w.ti = t / f.tiles_n3;  // row-block-major: rows of X' finish in order
    w.tj = t - w.ti * f.tiles_n3;
  } else {
    int i = 0;
    while ((i + 1) * (i + 2) / 2 <= t) ++i;  // lower-triangle row I holds tiles J = 0..I
    w.ti = i;
    w.tj = t - i * (i + 1) / 2;
  }
  w.ph = w.it * 3 + w.p;
  return w;
}

__device__ __forceinline__ int pair_fused_target(const FusedArgs& f, int q) {
  const int units = (q % 3 == 2) ? f.batch * f.tiles_m3 * f.tiles_n3 : f.batch * f.t_syrk;
  return (q / kFusedSlots + 1) * kPairEpiWarps * units;
}

// Bounded wait on a counter (phase or row block); `why` is the error code.
__device__ __forceinline__ bool wait_count_geq(const FusedArgs& f, const int* c, int target,
                                               volatile int* abort_flag) {
  unsigned long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if (ld_acquire_gpu(c) >= target) return true;
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
}

__device__ __forceinline__ bool pair_wait_phase(const FusedArgs& f, int q, int& done_upto,
                                                volatile int* abort_flag) {
  if (q < 0 || q <= done_upto) return true;
  if (!wait_count_geq(f, f.counters + (q % kFusedSlots), pair_fused_target(f, q), abort_flag))
    return false;
  done_upto = q;
  return true;
}

// Row block `row` of iteration it's X' (the B·X phase) complete.
__device__ __forceinline__ bool pair_wait_row(const FusedArgs& f, int it, int row,
                                              volatile int* abort_flag) {
  if (it < 0) return true;
  const int* c = f.rowdone + (it & 1) * f.tiles_m3 + row;
  return wait_count_geq(f, c, (it / 2 + 1) * kPairEpiWarps * f.batch * f.tiles_n3, abort_flag);
}

__global__ void __launch_bounds__(kThreads, 1)
    ns_fused_pair_kernel(const __grid_constant__ FusedMaps maps, const FusedArgs f) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* smemA = smem;
  uint8_t* smemB = smem + kPairStages * kPairTileA;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStageBytes);
  uint64_t* empty_bar = full_bar + kPairStages;
  uint64_t* accf_bar = empty_bar + kPairStages;
  uint64_t* acce_bar = accf_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
  __nv_bfloat16* sbuf = reinterpret_cast<__nv_bfloat16*>(smem + kPairStages * kPairStageBytes + 256);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader, 1 = peer
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int total = f.steps * f.units_iter;
  const int kb_n = (f.N + kBK - 1) / kBK;
  const int kb_m = (f.M + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], 8);
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
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the normalisation kernel's X0 is complete from here on

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int done_upto = -1;
      bool ok = true;
      for (int u = pair; u < total && ok; u += num_pairs) {
        const PairFusedUnit w = pair_fused_unit(f, u);
        if (w.p == 0) {
          if (!pair_wait_row(f, w.it - 1, w.ti, abort_flag) ||
              !pair_wait_row(f, w.it - 1, w.tj, abort_flag))
            break;
        } else {
          if (w.p == 2 && !pair_wait_phase(f, w.ph - 3, done_upto, abort_flag)) break;
          if (!pair_wait_phase(f, w.ph - 1, done_upto, abort_flag)) break;
        }
        fence_proxy_async_global();
        const CUtensorMap* ma = w.p == 0 ? &maps.xk[w.it & 1] : (w.p == 1 ? &maps.a : &maps.b);
        const CUtensorMap* mb = w.p == 0 ? &maps.xk[w.it & 1]
                                         : (w.p == 1 ? &maps.a : &maps.xmn[w.it & 1]);
        const int nkb = w.p == 0 ? kb_n : kb_m;
        const int arow = w.ti * kPairBM + static_cast<int>(rank) * 128;
        const int bcol = w.tj * kPairBN + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, f.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * kPairStageBytes);
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
          uint8_t* sa = smemA + stage * kPairTileA;
          uint8_t* sb = smemB + stage * kPairTileB;
          tma_load_3d_pair(sa, ma, fb, kb * kBK, arow, w.b);
          if (w.p == 2) {
            tma_load_3d_pair(sb, mb, fb, bcol, kb * kBK, w.b);
            tma_load_3d_pair(sb + kBK * 64 * 2, mb, fb, bcol + 64, kb * kBK, w.b);
          } else {
            tma_load_3d_pair(sb, mb, fb, kb * kBK, bcol, w.b);
          }
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    if (lane == 0) pdl_trigger();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc_k = make_idesc_bf16(kPairBM, kPairBN, 0, 0);
      constexpr uint32_t idesc_mn = make_idesc_bf16(kPairBM, kPairBN, 0, 1);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = pair; u < total && ok; u += num_pairs) {
        const int it = u / f.units_iter;
        const int r = u - it * f.units_iter;
        const int p = r < f.batch * f.t_syrk ? 0 : (r < 2 * f.batch * f.t_syrk ? 1 : 2);
        if (!mbar_wait_cluster(&acce_bar[acc], acc_phase ^ 1, abort_flag, f.err,
                               kErrWaitAccEmpty))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kPairBN;
        const int nkb = p == 0 ? kb_n : kb_m;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait_cluster(&full_bar[stage], phase, abort_flag, f.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smemA + stage * kPairTileA);
          const uint32_t sb = smem_u32(smemB + stage * kPairTileB);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = make_sdesc_sw128(sa + k * 32, 16, 1024);
            const uint64_t bdesc = p == 2 ? make_sdesc_sw128(sb + k * 2048, kBK * 64 * 2, 1024)
                                          : make_sdesc_sw128(sb + k * 32, 16, 1024);
            tc_mma_bf16_pair(d_tmem, adesc, bdesc, p == 2 ? idesc_mn : idesc_k,
                             (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit_pair(&empty_bar[stage], 0x3);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair(&accf_bar[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    __nv_bfloat16* wbuf = sbuf + (warp - 2) * (kEpiWarpBytes / 2);
    int acc = 0;
    uint32_t acc_phase = 0;
    int done_upto = -1;
    for (int u = pair; u < total; u += num_pairs) {
      const PairFusedUnit w = pair_fused_unit(f, u);
      bool ok = true;
      if (lane == 0) {
        if (w.p == 2) ok = pair_wait_phase(f, w.ph - 3, done_upto, abort_flag);
        if (ok && w.p >= 1) ok = pair_wait_phase(f, w.ph - 1, done_upto, abort_flag);
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      __syncwarp();
      if (!ok) break;
      FusedUnit fu;
      fu.it = w.it;
      fu.p = w.p;
      fu.ph = w.ph;
      fu.b = w.b;
      fu.ti = w.ti;
      fu.tj = w.tj;
      const GemmArgs g = fused_gemm_args(f, fu);
      const bool out_vec = ((reinterpret_cast<uintptr_t>(g.out) | (g.ld_out * 2)) & 15) == 0;
      const bool aux_vec = ((reinterpret_cast<uintptr_t>(g.aux) | (g.ld_aux * 2)) & 15) == 0;
      const uint32_t tacc = tmem_base + acc * kPairBN;
      const int row0w = w.ti * kPairBM + static_cast<int>(rank) * 128 + q * 32;
      const int col0 = w.tj * kPairBN;
      bool done;
      if (w.p == 0) {
        done = epilogue_tile<kSyrk>(g, tacc, q, row0w, col0, lane, out_vec, aux_vec,
                                    &accf_bar[acc], acc_phase, abort_flag, wbuf, &maps.so_a, w.b);
      } else if (w.p == 1) {
        done = epilogue_tile<kPoly>(g, tacc, q, row0w, col0, lane, out_vec, aux_vec,
                                    &accf_bar[acc], acc_phase, abort_flag, wbuf, &maps.so_b, w.b);
      } else {
        const CUtensorMap* so = w.it == f.steps - 1 ? &maps.so_out : &maps.so_x[(w.it + 1) & 1];
        done = epilogue_tile<kBX>(g, tacc, q, row0w, col0, lane, out_vec, aux_vec,
                                  &accf_bar[acc], acc_phase, abort_flag, wbuf, so, w.b);
      }
      if (!done) break;
      if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&acce_bar[acc]), 0));
      if (lane == 0) bulk_wait_all();
      __syncwarp();
      fence_proxy_async_global();
      __threadfence();
      __syncwarp();
      if (lane == 0) {
        red_release_gpu_add(f.counters + (w.ph % kFusedSlots), 1);
        if (w.p == 2) red_release_gpu_add(f.rowdone + (w.it & 1) * f.tiles_m3 + w.ti, 1);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync();  // all MMAs into either CTA's TMEM are complete and drained
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace fm
