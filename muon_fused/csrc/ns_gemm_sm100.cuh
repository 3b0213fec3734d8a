// Persistent tcgen05/TMEM GEMM for the three contractions of one
// Newton-Schulz iteration (reference: csrc/ns_gemm.cu:54-135 dispatches the
// same three products to sm_80 SYRK kernels and cuBLAS).
//
//   kSyrk  A  = X·Xᵀ                     lower-triangle tiles, mirrored store
//                                          (reference csrc/syrk_common.cuh:50-188, mode 0)
//   kPoly  B  = c·A·A + b·A  (off-diag)  lower-triangle tiles, mirrored store;
//          d  = a + diag(c·A·A + b·A)     kept in fp32
//                                          (reference csrc/syrk_common.cuh:147-157, mode 1,
//                                           which folds a·I into a bf16 B instead)
//   kBX    X' = d ⊙ X + B·X              full tiles; optional transposed store
//                                          (reference csrc/ns_gemm.cu:125-134, cuBLAS)
//
// Why the diagonal of B lives in fp32: B's diagonal is O(1) while the
// off-diagonal terms are small, so rounding the diagonal to bf16 dominates the
// iteration's error.  Keeping it in a separate fp32 vector and applying it in
// the kBX epilogue (d_i·X_ij in fp32) halves the relative error against an fp32
// Newton-Schulz.  B itself stays bit-symmetric (zero diagonal, each lower
// element written to both (r,c) and (c,r)).
//
// Structure (one CTA per SM, 6 warps):
//   warp 0      TMA producer: K-blocks of 64 bf16 (128 B rows, 128B swizzle)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..5  epilogue: tcgen05.ld TMEM -> registers -> fused math -> global
// Tile 128 (M) x 256 (N), kStages-deep smem ring, two TMEM accumulators of 256
// fp32 columns each so the epilogue of tile t overlaps the mainloop of t+1.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "fm_ptx.cuh"

namespace fm {

enum GemmMode : int { kSyrk = 0, kPoly = 1, kBX = 2 };

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kTileABytes = kBM * kBK * 2;  // 16 KB
constexpr int kTileBBytes = kBN * kBK * 2;  // 32 KB
constexpr int kStageBytes = kTileABytes + kTileBBytes;
constexpr int kTmemCols = 2 * kBN;  // two fp32 accumulators
// Epilogue staging in shared memory, per epilogue warp: two parities x
// {row-major, transposed} 32 x 32 bf16 blocks that TMA stores write out.
constexpr int kEpiBlock = 32 * 32;                  // elements of one block
constexpr int kEpiWarpBytes = 4 * kEpiBlock * 2;    // 8 KB per warp
constexpr int kEpiStageBytes = 4 * kEpiWarpBytes;   // 32 KB for the 4 epilogue warps
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align slack*/ + 256 /*barriers*/ +
                           kEpiStageBytes;

// Newton-Schulz quintic coefficients (reference muon_fused/ns_step.py:39).
constexpr float kNsA = 3.4445f;
constexpr float kNsB = -4.7750f;
constexpr float kNsC = 2.0315f;

struct GemmArgs {
  int M;          // output rows (m)
  int N;          // output columns: m for kSyrk/kPoly, n for kBX
  int K;          // reduction length: n for kSyrk, m otherwise
  int num_tiles;  // scheduled work units (batch x tiles x split)
  int tiles_n;    // kBX: column tiles per row block
  int tiles_m;    // kBX: row tiles per column block
  __nv_bfloat16* out;
  long long ld_out;
  const __nv_bfloat16* aux;  // kPoly: A (for b·A); kBX: X (for d ⊙ X)
  long long ld_aux;
  float* diag;        // kPoly: written; kBX: read
  int transpose_out;  // kBX: store X'ᵀ (ld_out is then the row stride of X'ᵀ)
  unsigned* err;      // device error word
  // Batched / split-K scheduling (CTA-pair kernel only; the single-CTA kernel
  // requires batch == 1 and split == 1).
  int batch;          // same-shape matrices in this launch (TMA dim 2 = matrix index)
  int tiles;          // output tiles per matrix
  int split;          // K-splits per tile
  int kb_per_split;   // K-blocks per split; the last split takes the remainder
  long long bs_out, bs_aux, bs_diag;  // per-matrix element strides
  float* partial;     // split > 1: fp32 partial tiles, 128 KB per (unit, CTA)
  int* counters;      // split > 1: arrivals per (matrix, tile, CTA), zero between uses
  int starve;         // self-test only: the producer issues no loads, so the MMA
                      // warp's bounded wait must run out and report kErrWaitFull
  int tma_out;        // 1: `out` is described by the kernel's store tensor map
                      // (16-byte aligned rows); the epilogue writes through it
};

// A GemmArgs whose pointers address matrix b of the batch.
__device__ __forceinline__ GemmArgs for_matrix(const GemmArgs& g, int b) {
  GemmArgs r = g;
  r.out = g.out + b * g.bs_out;
  r.aux = g.aux ? g.aux + b * g.bs_aux : nullptr;
  r.diag = g.diag ? g.diag + b * g.bs_diag : nullptr;
  return r;
}

// Number of 128x256 tiles intersecting the lower triangle of an m x m matrix.
__host__ __device__ inline int syrk_tile_count(int m) {
  const int mt = (m + kBM - 1) / kBM;
  int cnt = 0;
  for (int i = 0; i < mt; ++i) cnt += (i * kBM + kBM - 1) / kBN + 1;
  return cnt;
}

__device__ __forceinline__ void syrk_tile_coords(int t, int& ti, int& tj) {
  int i = 0;
  for (;; ++i) {
    const int c = (i * kBM + kBM - 1) / kBN + 1;
    if (t < c) break;
    t -= c;
  }
  ti = i;
  tj = t;
}

template <int MODE>
__device__ __forceinline__ void tile_coords(const GemmArgs& g, int t, int& ti, int& tj) {
  if constexpr (MODE == kBX) {
    // Column-block-major: concurrent CTAs share a few column blocks of X (the
    // larger operand, streamed once) and sweep all row blocks of B (m x m,
    // the smaller one, which stays in L2).
    tj = t / g.tiles_m;
    ti = t - tj * g.tiles_m;
  } else {
    syrk_tile_coords(t, ti, tj);
  }
}

__device__ __forceinline__ uint4 pack8_bf16(const float* v) {
  uint4 u;
  __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]);
  __nv_bfloat162 h1 = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 h2 = __floats2bfloat162_rn(v[4], v[5]);
  __nv_bfloat162 h3 = __floats2bfloat162_rn(v[6], v[7]);
  u.x = *reinterpret_cast<uint32_t*>(&h0);
  u.y = *reinterpret_cast<uint32_t*>(&h1);
  u.z = *reinterpret_cast<uint32_t*>(&h2);
  u.w = *reinterpret_cast<uint32_t*>(&h3);
  return u;
}

__device__ __forceinline__ void unpack8_bf16(uint4 u, float* v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
    float2 f = __bfloat1622float2(h);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Load 32 bf16 values of one row starting at column c0 (masked by ncols).
// `vec` says rows are 16-byte aligned (base and row stride), allowing 16-byte loads.
__device__ __forceinline__ void load_row32(const __nv_bfloat16* rowp, int c0, int ncols, bool vec,
                                           float (&v)[32]) {
  if (vec && c0 + 32 <= ncols) {
    const uint4* p = reinterpret_cast<const uint4*>(rowp + c0);
#pragma unroll
    for (int q = 0; q < 4; ++q) unpack8_bf16(__ldg(p + q), v + 8 * q);
  } else {
#pragma unroll
    for (int k = 0; k < 32; ++k)
      v[k] = (c0 + k < ncols) ? __bfloat162float(rowp[c0 + k]) : 0.f;
  }
}

// Raw (still packed bf16) form of load_row32, so a chunk can be fetched one
// step ahead of its use without spending 32 registers on it.
__device__ __forceinline__ void load_raw32(const __nv_bfloat16* rowp, int c0, int ncols, bool vec,
                                           uint4 (&r)[4]) {
  if (vec && c0 + 32 <= ncols) {
    const uint4* p = reinterpret_cast<const uint4*>(rowp + c0);
#pragma unroll
    for (int q = 0; q < 4; ++q) r[q] = __ldg(p + q);
  } else {
    uint16_t h[32];
#pragma unroll
    for (int k = 0; k < 32; ++k)
      h[k] = (c0 + k < ncols) ? __bfloat16_as_ushort(rowp[c0 + k]) : static_cast<uint16_t>(0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      r[q].x = h[8 * q + 0] | (static_cast<uint32_t>(h[8 * q + 1]) << 16);
      r[q].y = h[8 * q + 2] | (static_cast<uint32_t>(h[8 * q + 3]) << 16);
      r[q].z = h[8 * q + 4] | (static_cast<uint32_t>(h[8 * q + 5]) << 16);
      r[q].w = h[8 * q + 6] | (static_cast<uint32_t>(h[8 * q + 7]) << 16);
    }
  }
}

// Mirror of a lower-triangle chunk: value (row, c) also goes to (c, row) for
// c < row.  Lanes hold consecutive rows, so each store instruction writes 64
// contiguous bytes of row c.
__device__ __forceinline__ void store_mirror32(__nv_bfloat16* out, long long ld, int c0, int ncols,
                                               int row, const float (&v)[32]) {
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const int col = c0 + k;
    if (col < row && col < ncols) out[static_cast<long long>(col) * ld + row] = __float2bfloat16_rn(v[k]);
  }
}

// Store 32 values of one row (row-major, masked by ncols and an optional
// lower-triangle predicate col <= row).
__device__ __forceinline__ void store_row32(__nv_bfloat16* rowp, int c0, int ncols, int row,
                                            bool lower_only, bool vec, const float (&v)[32]) {
  const bool full = vec && (c0 + 32 <= ncols) && (!lower_only || c0 + 31 <= row);
  if (full) {
    uint4* p = reinterpret_cast<uint4*>(rowp + c0);
#pragma unroll
    for (int q = 0; q < 4; ++q) p[q] = pack8_bf16(v + 8 * q);
  } else {
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      const int c = c0 + k;
      if (c < ncols && (!lower_only || c <= row)) rowp[c] = __float2bfloat16_rn(v[k]);
    }
  }
}

// Per-warp shared buffer for 32 x 32 transposed stores of the direct-store
// fallback: rows of 34 bf16 (17 words, odd, so the row-wise 4-byte writes hit
// 32 distinct banks).  It lives in the warp's staging area.
constexpr int kTPitch = 34;

// out[(c0 + l) * ld + row0w + j] = v_j[l] for the warp's 32 rows j and the
// chunk's 32 columns l: the chunk goes through shared memory so that each lane
// writes one output row of 64 bytes as four 16-byte stores (instead of 32
// two-byte stores per lane).  All 32 rows and columns must be in bounds and
// the output rows 16-byte aligned.
__device__ __forceinline__ void store_transposed32(__nv_bfloat16* out, long long ld, int row0w,
                                                   int c0, int lane, __nv_bfloat16* tb,
                                                   const float (&v)[32]) {
  __syncwarp();  // the previous chunk's reads are done
  uint32_t* trow = reinterpret_cast<uint32_t*>(tb + lane * kTPitch);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
    trow[k] = *reinterpret_cast<uint32_t*>(&h);
  }
  __syncwarp();
  __align__(16) __nv_bfloat16 o[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) o[j] = tb[j * kTPitch + lane];
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(c0 + lane) * ld + row0w);
#pragma unroll
  for (int q = 0; q < 4; ++q) dst[q] = reinterpret_cast<const uint4*>(o)[q];
}

// Staging of one 32 x 32 chunk for a TMA store.  Lane r holds row r of the
// chunk in v.  Row-major: row r is 64 contiguous bytes.  Transposed: element
// (r, k) goes to (k, r), so each store instruction of the warp writes 64
// contiguous bytes.  Symmetric: the block on the diagonal of a SYRK output,
// built from its lower triangle only (what the direct-store path writes).
__device__ __forceinline__ void stage_rows32(__nv_bfloat16* blk, int lane, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(blk + lane * 32);
#pragma unroll
  for (int q = 0; q < 4; ++q) d[q] = pack8_bf16(v + 8 * q);
}
__device__ __forceinline__ void stage_cols32(__nv_bfloat16* blk, int lane, const float (&v)[32]) {
#pragma unroll
  for (int k = 0; k < 32; ++k) blk[k * 32 + lane] = __float2bfloat16_rn(v[k]);
}
__device__ __forceinline__ void stage_sym32(__nv_bfloat16* blk, int lane, const float (&v)[32]) {
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v[k]);
    if (k <= lane) blk[lane * 32 + k] = h;
    if (k < lane) blk[k * 32 + lane] = h;
  }
}

// Number of 32-column chunks of a tile row block that warp rows row0w.. store:
// a prefix (columns below N; for the SYRK modes also at or left of the warp's
// last row).
template <int MODE, int TBN = kBN>
__device__ __forceinline__ int epilogue_chunks(const GemmArgs& g, int row0w, int col0) {
  int col_end = min(g.N, col0 + TBN);
  if constexpr (MODE != kBX) col_end = min(col_end, row0w + 32);
  return row0w < g.M ? max(0, (col_end - col0 + 31) / 32) : 0;
}

// Split-K partial layout for one CTA's 128 x 256 fp32 accumulator:
// element (row 32q + lane, column 32c + k) at ((q*8 + c)*32 + k)*32 + lane,
// so each warp store / load instruction covers 128 contiguous bytes.
constexpr int kPartialFloats = 128 * 256;
__device__ __forceinline__ int partial_index(int q, int c, int k, int lane) {
  return ((q * 8 + c) * 32 + k) * 32 + lane;
}

// Split-K, first half of the epilogue: wait for this split's accumulator and
// write its needed chunks to `dst` (this unit's partial slot).  Returns false
// if the wait gave up.
template <int MODE>
__device__ __forceinline__ bool stash_partial(const GemmArgs& g, uint32_t tmem_acc, int q, int row0w,
                                              int col0, int lane, float* dst, uint64_t* accf_bar,
                                              uint32_t acc_phase, volatile int* abort_flag) {
  const int nc = epilogue_chunks<MODE>(g, row0w, col0);
  if (!mbar_wait(accf_bar, acc_phase, abort_flag, g.err, kErrWaitAccFull)) return false;
  tc_fence_after();
#pragma unroll 1
  for (int c = 0; c < nc; ++c) {
    float v[32];
    tmem_ld_32x32b_x32(tmem_acc + c * 32 + (static_cast<uint32_t>(q * 32) << 16), v);
#pragma unroll
    for (int k = 0; k < 32; ++k) __stcg(dst + partial_index(q, c, k, lane), v[k]);
  }
  tc_fence_before();
  __syncwarp();
  return true;
}

// Epilogue of one output tile for one warp: lane quarter q holds rows
// row0w .. row0w+31; the tile's columns start at col0.
//   FROM_PARTIALS = false: values come from the TMEM accumulator at tmem_acc,
//     after waiting on accf_bar (parity acc_phase); returns false if that
//     wait gave up.  Shared by the 1-CTA, 2-CTA and persistent kernels.
//   FROM_PARTIALS = true: values are the sum, in split order, of `split`
//     fp32 partials starting at `parts` (stride kPartialFloats) — the
//     last-arriving split of a split-K tile runs this.
// Stores: with g.tma_out, each 32 x 32 chunk is staged in the warp's shared
// buffers `sbuf` (8 KB: two parities x {row-major, transposed}) and written
// by TMA tile stores through `tm_out` at matrix index `bz`; lane 0 issues
// them and keeps at most one older chunk's stores in flight, so the warp
// moves on while the copies drain.  Otherwise every lane stores its own row
// (unaligned outputs).  The caller waits for outstanding stores
// (bulk_wait_all) before the results are consumed or the CTA exits.
template <int MODE, bool FROM_PARTIALS = false, int TBN = kBN>
__device__ __forceinline__ bool epilogue_tile(const GemmArgs& g, uint32_t tmem_acc, int q,
                                              int row0w, int col0, int lane, bool out_vec,
                                              bool aux_vec, uint64_t* accf_bar, uint32_t acc_phase,
                                              volatile int* abort_flag,
                                              __nv_bfloat16* sbuf, const CUtensorMap* tm_out,
                                              int bz, const float* parts = nullptr,
                                              int split = 1) {
  const int row = row0w + lane;
  const bool row_ok = row < g.M;
  const __nv_bfloat16* aux_row = g.aux + static_cast<long long>(row) * g.ld_aux;
  const int nc = epilogue_chunks<MODE, TBN>(g, row0w, col0);
  const bool use_tma = g.tma_out != 0;
  // The epilogue operand (A for kPoly, X for kBX) does not depend on the
  // accumulator: fetch the first chunk before waiting for the MMAs and each
  // next chunk while the current one is processed.
  uint4 araw[4], anext[4];
  if constexpr (MODE != kSyrk) {
    if (nc > 0 && row_ok) load_raw32(aux_row, col0, g.N, aux_vec, araw);
  }
  float dval = 0.f;
  if constexpr (MODE == kBX) dval = row_ok ? g.diag[row] : 0.f;
  if constexpr (!FROM_PARTIALS) {
    if (!mbar_wait(accf_bar, acc_phase, abort_flag, g.err, kErrWaitAccFull)) return false;
    tc_fence_after();
  }
#pragma unroll 1
  for (int c = 0; c < nc; ++c) {
    const int c0 = col0 + c * 32;
    if constexpr (MODE != kSyrk) {
      if (c + 1 < nc && row_ok) load_raw32(aux_row, c0 + 32, g.N, aux_vec, anext);
    }
    float v[32];
    if constexpr (FROM_PARTIALS) {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = __ldcg(parts + partial_index(q, c, k, lane));
      for (int sp = 1; sp < split; ++sp) {
        const float* ps = parts + static_cast<long long>(sp) * kPartialFloats;
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] += __ldcg(ps + partial_index(q, c, k, lane));
      }
    } else {
      tmem_ld_32x32b_x32(tmem_acc + c * 32 + (static_cast<uint32_t>(q * 32) << 16), v);
    }
    if constexpr (MODE == kPoly) {
      if (row_ok) {
        float av[32];
#pragma unroll
        for (int k = 0; k < 4; ++k) unpack8_bf16(araw[k], av + 8 * k);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          float x = fmaf(kNsC, v[k], kNsB * av[k]);
          if (c0 + k == row) {
            g.diag[row] = x + kNsA;
            x = 0.f;
          }
          v[k] = x;
        }
      }
    }
    if constexpr (MODE == kBX) {
      float xv[32];
#pragma unroll
      for (int k = 0; k < 4; ++k) unpack8_bf16(araw[k], xv + 8 * k);
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = fmaf(dval, xv[k], v[k]);
    }
    if (use_tma) {
      __nv_bfloat16* bd = sbuf + (c & 1) * 2 * kEpiBlock;
      __nv_bfloat16* bt = bd + kEpiBlock;
      if (lane == 0) bulk_wait_read<1>();  // chunk c-2's stores have read this parity
      __syncwarp();
      bool st_rows = true, st_cols = false;
      if constexpr (MODE != kBX) {
        if (c0 == row0w) {
          stage_sym32(bd, lane, v);  // diagonal block, symmetric
        } else {
          stage_rows32(bd, lane, v);  // strictly below the diagonal: direct + mirror
          stage_cols32(bt, lane, v);
          st_cols = true;
        }
      } else if (g.transpose_out) {
        stage_cols32(bt, lane, v);
        st_rows = false;
        st_cols = true;
      } else {
        stage_rows32(bd, lane, v);
      }
      fence_proxy_async_shared();
      __syncwarp();
      if (lane == 0) {
        if (st_rows) tma_store_3d(tm_out, bd, c0, row0w, bz);
        if (st_cols) tma_store_3d(tm_out, bt, row0w, c0, bz);
        bulk_commit();
      }
    } else {
      // All 32 rows and columns of this chunk in bounds (warp-uniform): the
      // column-wise stores (mirror, transposed output) can go through smem.
      const bool whole = row0w + 31 < g.M && c0 + 31 < g.N && out_vec;
      if constexpr (MODE != kBX) {
        if (row_ok) store_row32(g.out + row * g.ld_out, c0, g.N, row, true, out_vec, v);
        if (whole && c0 + 31 < row0w) {  // chunk strictly below the diagonal
          store_transposed32(g.out, g.ld_out, row0w, c0, lane, sbuf, v);
        } else if (row_ok) {
          store_mirror32(g.out, g.ld_out, c0, g.N, row, v);
        }
      } else {
        if (g.transpose_out) {
          if (whole) {
            store_transposed32(g.out, g.ld_out, row0w, c0, lane, sbuf, v);
          } else if (row_ok) {
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const int col = c0 + k;
              if (col < g.N)
                g.out[static_cast<long long>(col) * g.ld_out + row] = __float2bfloat16_rn(v[k]);
            }
          }
        } else if (row_ok) {
          store_row32(g.out + row * g.ld_out, c0, g.N, row, false, out_vec, v);
        }
      }
    }
    if constexpr (MODE != kSyrk) {
#pragma unroll
      for (int k = 0; k < 4; ++k) araw[k] = anext[k];
    }
  }
  if constexpr (!FROM_PARTIALS) tc_fence_before();
  __syncwarp();
  return true;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    ns_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO, const GemmArgs g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 128B-swizzled TMA destinations need 1024-byte alignment.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* smemA = smem;
  uint8_t* smemB = smem + kStages * kTileABytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* accf_bar = empty_bar + kStages;  // accumulator ready  [2]
  uint64_t* acce_bar = accf_bar + 2;         // accumulator drained [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
  // per-warp epilogue staging buffers, after the 256-byte barrier block
  __nv_bfloat16* sbuf = reinterpret_cast<__nv_bfloat16*>(smem + kStages * kStageBytes + 256);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = (g.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], 4);  // one arrive per epilogue warp
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the previous kernel's outputs are complete from here on

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !g.starve) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < g.num_tiles && ok; t += gridDim.x) {
        int ti, tj;
        tile_coords<MODE>(g, t, ti, tj);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, g.err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], kStageBytes);
          uint8_t* sa = smemA + stage * kTileABytes;
          uint8_t* sb = smemB + stage * kTileBBytes;
          tma_load_3d(sa, &tmA, &full_bar[stage], kb * kBK, ti * kBM, 0);
          if constexpr (MODE == kBX) {
            // B operand is X (K = rows, N = contiguous columns): four MN-major
            // boxes of 64 columns x 64 rows, 8 KB apart.
#pragma unroll
            for (int q = 0; q < 4; ++q)
              tma_load_3d(sb + q * (kBK * 64 * 2), &tmB, &full_bar[stage], tj * kBN + q * 64,
                          kb * kBK, 0);
          } else {
            tma_load_3d(sb, &tmB, &full_bar[stage], kb * kBK, tj * kBN, 0);
            tma_load_3d(sb + kTileABytes, &tmB, &full_bar[stage], kb * kBK, tj * kBN + kBM, 0);
          }
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    if (lane == 0) pdl_trigger();  // all loads issued: the next kernel may launch
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kBM, kBN, 0, MODE == kBX ? 1 : 0);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < g.num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1, abort_flag, g.err, kErrWaitAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, g.err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smemA + stage * kTileABytes);
          const uint32_t sb = smem_u32(smemB + stage * kTileBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // K-major SW128: advance 16 elements = 32 bytes inside the swizzle row.
            const uint64_t adesc = make_sdesc_sw128(sa + k * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (MODE == kBX) {
              // MN-major SW128: 16 K-rows = 2048 bytes; LBO = 8 KB between
              // 64-column chunks, SBO = 1 KB between 8-row groups.
              bdesc = make_sdesc_sw128(sb + k * 2048, kBK * 64 * 2, 1024);
            } else {
              bdesc = make_sdesc_sw128(sb + k * 32, 16, 1024);
            }
            tc_mma_bf16(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          tc_commit(&empty_bar[stage]);  // frees the smem stage when these MMAs finish
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&accf_bar[acc]);  // accumulator complete
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    // 16-byte vector access only when base pointer and row stride allow it
    const bool out_vec = ((reinterpret_cast<uintptr_t>(g.out) | (g.ld_out * 2)) & 15) == 0;
    const bool aux_vec = ((reinterpret_cast<uintptr_t>(g.aux) | (g.ld_aux * 2)) & 15) == 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < g.num_tiles; t += gridDim.x) {
      int ti, tj;
      tile_coords<MODE>(g, t, ti, tj);
      if (!epilogue_tile<MODE>(g, tmem_base + acc * kBN, q, ti * kBM + q * 32, tj * kBN, lane,
                               out_vec, aux_vec, &accf_bar[acc], acc_phase, abort_flag,
                               sbuf + (warp - 2) * (kEpiWarpBytes / 2), &tmO, 0))
        break;
      if (lane == 0) mbar_arrive(&acce_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait_all();  // TMA stores done before the CTA exits
    __syncwarp();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace fm
