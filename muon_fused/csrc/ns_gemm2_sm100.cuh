// CTA-pair (tcgen05 cta_group::2) version of the Newton-Schulz GEMMs.
//
// Same three modes and epilogues as ns_gemm_sm100.cuh, on 256 x 256 output
// tiles computed by a 2-CTA cluster:
//   * each CTA TMA-loads its own 128 rows of the A operand and its own half
//     (128 rows / columns) of the B operand into its own shared memory — no
//     multicast, so per CTA a K-block costs 32 KB instead of 48 KB;
//   * the leader (even) CTA issues one M=256, N=256 MMA per K=16 step that
//     reads both CTAs' shared memory and accumulates into both CTAs' TMEM
//     (rows 0..127 in the leader, 128..255 in the peer);
//   * stage release and "accumulator ready" are tcgen05.commit multicasts to
//     both CTAs; "accumulator drained" is 4 local + 4 remote warp arrivals on
//     the leader's barrier.
// Six 32 KB stages (192 KB) keep about 3000 MMA cycles of loads in flight.
//
// Scheduling: a work unit is (matrix b of the batch, output tile, K-split s);
// pairs walk the units persistently.  With split > 1 each split stashes its
// fp32 accumulator half in the workspace; the last split to arrive (per tile
// and CTA, counted with an atomic) sums all splits in split order — so the
// result does not depend on arrival order — and runs the fused epilogue.
#pragma once
#include "ns_gemm_sm100.cuh"

namespace fm {

constexpr int kPairBM = 256;  // rows of a pair tile (128 per CTA)
constexpr int kPairBN = 256;  // columns of a pair tile
constexpr int kPairStages = 6;
constexpr int kPairTileA = 128 * kBK * 2;  // 16 KB: this CTA's A rows
constexpr int kPairTileB = 128 * kBK * 2;  // 16 KB: this CTA's half of B
constexpr int kPairStageBytes = kPairTileA + kPairTileB;
constexpr int kPairSmemBytes = kPairStages * kPairStageBytes + 1024 + 256 + kEpiStageBytes;

// Lower-triangle 256 x 256 tiles of an m x m matrix: T(T+1)/2, T = ceil(m/256).
__host__ __device__ inline int syrk_pair_tile_count(int m) {
  const int t = (m + kPairBM - 1) / kPairBM;
  return t * (t + 1) / 2;
}

template <int MODE>
__device__ __forceinline__ void pair_tile_coords(const GemmArgs& g, int t, int& ti, int& tj) {
  if constexpr (MODE == kBX) {
    tj = t / g.tiles_m;  // column-block-major, as in the 1-CTA kernel
    ti = t - tj * g.tiles_m;
  } else {
    int i = 0;
    while ((i + 1) * (i + 2) / 2 <= t) ++i;  // row I holds tiles J = 0..I
    ti = i;
    tj = t - i * (i + 1) / 2;
  }
}

struct PairUnit {
  int b, ti, tj, s, kb0, kb1, tile;
};

template <int MODE>
__device__ __forceinline__ PairUnit pair_unit(const GemmArgs& g, int u, int num_kb) {
  PairUnit w;
  const int per_matrix = g.tiles * g.split;
  w.b = u / per_matrix;
  const int r = u - w.b * per_matrix;
  w.tile = r / g.split;
  w.s = r - w.tile * g.split;
  pair_tile_coords<MODE>(g, w.tile, w.ti, w.tj);
  w.kb0 = w.s * g.kb_per_split;
  w.kb1 = (w.s == g.split - 1) ? num_kb : w.kb0 + g.kb_per_split;
  return w;
}

#ifdef FM_TRACE
// Development timeline (built only with -DFM_TRACE): per GEMM mode and pair,
// slot 0 = start of work, then per unit k: 1+3k MMA start, 2+3k MMAs issued,
// 3+3k epilogue done (leader CTA); slot 38 = kernel entry, 39 = kernel exit.
// Read with fm_trace_read.
__device__ unsigned long long g_fm_trace[3][128][40];
#define FM_TRACE_MARK(slot)                                                       \
  do {                                                                            \
    if ((slot) < 38) g_fm_trace[MODE][pair][(slot)] = globaltimer();              \
  } while (0)
#define FM_TRACE_EDGE(slot) g_fm_trace[MODE][pair][(slot)] = globaltimer()
#else
#define FM_TRACE_MARK(slot) \
  do {                      \
  } while (0)
#define FM_TRACE_EDGE(slot) \
  do {                      \
  } while (0)
#endif

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    ns_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmO, const GemmArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* smemA = smem;
  uint8_t* smemB = smem + kPairStages * kPairTileA;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kPairStages * kPairStageBytes);
  uint64_t* empty_bar = full_bar + kPairStages;
  uint64_t* accf_bar = empty_bar + kPairStages;  // accumulator ready  [2]
  uint64_t* acce_bar = accf_bar + 2;             // accumulator drained [2] (leader's used)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
  // per-warp epilogue staging buffers, after the 256-byte barrier block
  __nv_bfloat16* sbuf = reinterpret_cast<__nv_bfloat16*>(smem + kPairStages * kPairStageBytes + 256);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0 = leader, 1 = peer
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_kb = (g.K + kBK - 1) / kBK;
  if (threadIdx.x == 0 && rank == 0) FM_TRACE_EDGE(38);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full_bar[s], 1);   // leader: its own expect_tx arrival (+ both CTAs' bytes)
      mbar_init(&empty_bar[s], 1);  // both: one multicast commit per use
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);  // both: one multicast commit per tile
      mbar_init(&acce_bar[a], 8);  // leader: 4 epilogue warps of each CTA
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs are complete from here on
  if (threadIdx.x == 0 && rank == 0) FM_TRACE_MARK(0);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < g.num_tiles && ok; t += num_pairs) {
        const PairUnit w = pair_unit<MODE>(g, t, num_kb);
        const int arow = w.ti * kPairBM + static_cast<int>(rank) * 128;  // this CTA's A rows
        const int bcol = w.tj * kPairBN + static_cast<int>(rank) * 128;  // this CTA's half of B
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, g.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * kPairStageBytes);
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
          uint8_t* sa = smemA + stage * kPairTileA;
          uint8_t* sb = smemB + stage * kPairTileB;
          tma_load_3d_pair(sa, &tmA, fb, kb * kBK, arow, w.b);
          if constexpr (MODE == kBX) {
            // X columns bcol..bcol+127: two MN-major boxes of 64 columns x 64 rows
            tma_load_3d_pair(sb, &tmB, fb, bcol, kb * kBK, w.b);
            tma_load_3d_pair(sb + kBK * 64 * 2, &tmB, fb, bcol + 64, kb * kBK, w.b);
          } else {
            tma_load_3d_pair(sb, &tmB, fb, kb * kBK, bcol, w.b);
          }
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    if (lane == 0) pdl_trigger();  // all loads issued: the next kernel may launch
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kPairBM, kPairBN, 0, MODE == kBX ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      int nunit = 0;  // trace index only
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < g.num_tiles && ok; t += num_pairs) {
        if (!mbar_wait_cluster(&acce_bar[acc], acc_phase ^ 1, abort_flag, g.err,
                               kErrWaitAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const PairUnit w = pair_unit<MODE>(g, t, num_kb);
        const uint32_t d_tmem = tmem_base + acc * kPairBN;
        FM_TRACE_MARK(1 + 3 * nunit);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_cluster(&full_bar[stage], phase, abort_flag, g.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smemA + stage * kPairTileA);
          const uint32_t sb = smem_u32(smemB + stage * kPairTileB);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = make_sdesc_sw128(sa + k * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (MODE == kBX) {
              bdesc = make_sdesc_sw128(sb + k * 2048, kBK * 64 * 2, 1024);
            } else {
              bdesc = make_sdesc_sw128(sb + k * 32, 16, 1024);
            }
            tc_mma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb > w.kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit_pair(&empty_bar[stage], 0x3);  // frees this stage in both CTAs
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit_pair(&accf_bar[acc], 0x3);  // accumulator complete in both CTAs
        FM_TRACE_MARK(2 + 3 * nunit);
        ++nunit;
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const bool out_vec = ((reinterpret_cast<uintptr_t>(g.out) | (g.ld_out * 2)) & 15) == 0;
    const bool aux_vec = ((reinterpret_cast<uintptr_t>(g.aux) | (g.ld_aux * 2)) & 15) == 0;
    volatile int* last_flag = abort_flag + 1;  // smem word shared by the epilogue warps
    int acc = 0;
    int nunit = 0;  // trace index only
    uint32_t acc_phase = 0;
    for (int t = pair; t < g.num_tiles; t += num_pairs) {
      const PairUnit w = pair_unit<MODE>(g, t, num_kb);
      const GemmArgs gb = for_matrix(g, w.b);
      const int row0w = w.ti * kPairBM + static_cast<int>(rank) * 128 + q * 32;
      const int col0 = w.tj * kPairBN;
      const uint32_t tacc = tmem_base + acc * kPairBN;
      const uint32_t acce_remote = mapa_shared(smem_u32(&acce_bar[acc]), 0);
      if (g.split == 1) {
        if (!epilogue_tile<MODE>(gb, tacc, q, row0w, col0, lane, out_vec, aux_vec, &accf_bar[acc],
                                 acc_phase, abort_flag, sbuf + (warp - 2) * (kEpiWarpBytes / 2),
                                 &tmO, w.b))
          break;
        if (lane == 0) mbar_arrive_remote(acce_remote);
        if (lane == 0 && q == 2 && rank == 0) FM_TRACE_MARK(3 + 3 * nunit);
        ++nunit;
      } else {
        // this (matrix, tile, CTA half)'s partial slots, split 0 first
        const long long slot = (static_cast<long long>(w.b) * g.tiles + w.tile) * 2 + rank;
        float* parts = g.partial + slot * g.split * static_cast<long long>(kPartialFloats);
        // A failed wait still goes through the three epilogue barriers below
        // (so no warp is left waiting at one) and then leaves the loop.
        const bool ok = stash_partial<MODE>(gb, tacc, q, row0w, col0, lane,
                                            parts + static_cast<long long>(w.s) * kPartialFloats,
                                            &accf_bar[acc], acc_phase, abort_flag);
        if (ok && lane == 0) mbar_arrive_remote(acce_remote);  // TMEM free for the next unit
        __threadfence();
        epilogue_bar_sync();
        if (threadIdx.x == 64) {  // first epilogue thread decides for all four warps
          if (*abort_flag) {
            *last_flag = 2;  // a wait failed (it raised the flag before the barrier)
          } else {
            const int prev = atomicAdd(&g.counters[slot], 1);
            const int last = prev == g.split - 1;
            if (last) g.counters[slot] = 0;  // ready for the next launch using this slot
            *last_flag = last;
          }
        }
        epilogue_bar_sync();
        const int verdict = *last_flag;
        epilogue_bar_sync();  // everyone has read the verdict before it is rewritten
        if (verdict == 2) break;
        const bool last = verdict == 1;
        if (last) {
          __threadfence();
          epilogue_tile<MODE, true>(gb, 0, q, row0w, col0, lane, out_vec, aux_vec, nullptr, 0,
                                    abort_flag, sbuf + (warp - 2) * (kEpiWarpBytes / 2), &tmO,
                                    w.b, parts, g.split);
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait_all();  // TMA stores done before the CTA exits
    __syncwarp();
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync();  // all MMAs into either CTA's TMEM are complete and drained
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && rank == 0) FM_TRACE_EDGE(39);
}

}  // namespace fm
