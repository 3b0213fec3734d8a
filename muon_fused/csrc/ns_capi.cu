// Host orchestration and the C ABI (include/fused_muon.h).
//
// Replaces the reference's host side: csrc/torch_binding.cu (cast, transpose,
// normalise, step loop) and csrc/ns_gemm.cu (workspace layout, GEMM dispatch).
// One Newton-Schulz call is 2 bandwidth kernels + 3 tcgen05 GEMMs per step,
// all on the caller's stream with no host synchronisation.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "../../include/fused_muon.h"
#include "ns_gemm2_sm100.cuh"
#include "ns_gemm_sm100.cuh"
#include "ns_fused_sm100.cuh"
#include "ns_fused2_sm100.cuh"
#include "muon_elementwise.cuh"
#include "ns_prep.cuh"

namespace fm {

__device__ unsigned g_device_error;  // first timed-out wait code, see fm_ptx.cuh

namespace {

thread_local char t_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

#define FM_CUDA(call)                                                                   \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return fail(FM_E_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                  __FILE__, __LINE__);                                                  \
  } while (0)

constexpr int kMaxDevices = 64;

// `ready` is published with release semantics after every other field is
// written, and read with acquire semantics on the lock-free fast path.
struct DeviceState {
  std::atomic<bool> ready{false};
  int sm_count = 0;
  unsigned* err_word = nullptr;
};
DeviceState g_dev[kMaxDevices];
std::mutex g_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

inline long long round_up(long long x, long long a) { return (x + a - 1) / a * a; }

// Counter area of the persistent kernels in the workspace: the phase ring, then
// 2 x T row-block counters of the CTA-pair kernel (T <= kMaxPairRows).
constexpr int kPhaseBytes = 1024;
constexpr int kRowdoneOffset = 16;  // ints
constexpr int kMaxPairRows = (kPhaseBytes / 4 - kRowdoneOffset) / 2;

// Optional per-stage timing for benchmarks (fm_stage_timing / fm_stage_times):
// when enabled, each kernel launch of this thread is bracketed by CUDA events
// on its stream; the pairs are resolved and summed per stage on request.
// 0 GEMM1 (X·Xᵀ), 1 GEMM2 (poly), 2 GEMM3 (B·X), 3 prep kernels, 4 persistent NS kernel
constexpr int kStages4 = 5;
struct StageTimer {
  bool on = false;
  std::vector<cudaEvent_t> pool;
  size_t used = 0;
  std::vector<std::pair<int, size_t>> marks;  // (stage, index of start event)
};
thread_local StageTimer t_timer;

int timer_event(cudaEvent_t* ev) {
  StageTimer& T = t_timer;
  if (T.used == T.pool.size()) {
    cudaEvent_t e;
    FM_CUDA(cudaEventCreate(&e));
    T.pool.push_back(e);
  }
  *ev = T.pool[T.used++];
  return FM_OK;
}

// Records the start event of a stage launch; returns the start index or -1.
long long timer_begin(int stage, cudaStream_t st) {
  if (!t_timer.on) return -1;
  cudaEvent_t e;
  if (timer_event(&e)) return -1;
  cudaEventRecord(e, st);
  t_timer.marks.push_back({stage, t_timer.used - 1});
  return static_cast<long long>(t_timer.used - 1);
}

void timer_end(long long start, cudaStream_t st) {
  if (start < 0) return;
  cudaEvent_t e;
  if (timer_event(&e)) return;
  cudaEventRecord(e, st);
}

// Per-device set-up: SM count, smem opt-in for the GEMM kernels, address of
// the device error word.  Runs once per device, with that device current.
int device_state(DeviceState** out) {
  int dev = 0;
  FM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(FM_E_DEVICE, "device index %d out of range", dev);
  DeviceState& s = g_dev[dev];
  if (!s.ready.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!s.ready.load(std::memory_order_relaxed)) {
      int major = 0, minor = 0;
      FM_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
      FM_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
      if (major != 10 || minor != 0)
        return fail(FM_E_DEVICE, "fused_muon kernels are built for sm_100a; device %d is sm_%d%d",
                    dev, major, minor);
      FM_CUDA(cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, dev));
      FM_CUDA(cudaFuncSetAttribute(ns_gemm_kernel<kSyrk>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
      FM_CUDA(cudaFuncSetAttribute(ns_gemm_kernel<kPoly>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
      FM_CUDA(cudaFuncSetAttribute(ns_gemm_kernel<kBX>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
      FM_CUDA(cudaFuncSetAttribute(ns_gemm_pair_kernel<kSyrk>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmemBytes));
      FM_CUDA(cudaFuncSetAttribute(ns_gemm_pair_kernel<kPoly>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmemBytes));
      FM_CUDA(cudaFuncSetAttribute(ns_gemm_pair_kernel<kBX>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmemBytes));
      FM_CUDA(cudaFuncSetAttribute(ns_fused_kernel<256>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   FusedCfg<256>::kSmem));
      FM_CUDA(cudaFuncSetAttribute(ns_fused_kernel<128>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   FusedCfg<128>::kSmem));
      FM_CUDA(cudaFuncSetAttribute(ns_fused_pair_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kPairSmemBytes));
      FM_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&s.err_word), g_device_error));
      if (!g_encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        FM_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn)
          return fail(FM_E_CUDA, "cuTensorMapEncodeTiled entry point not found");
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      }
      s.ready.store(true, std::memory_order_release);
    }
  }
  *out = &s;
  return FM_OK;
}

// 3-D bf16 tensor map over `batch` row-major rows x cols matrices with row
// stride ld and matrix stride bstride (elements); box = box_cols (inner) x
// box_rows x 1, zero fill out of bounds.  Operand maps use the 128-byte
// swizzle of the MMA's shared-memory layout; store maps none.
int make_map(CUtensorMap* map, const void* base, long long batch, long long rows, long long cols,
             long long ld, long long bstride, int box_cols, int box_rows,
             CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  if (batch == 1) bstride = round_up(rows * ld, 8);
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * 2) % 16 != 0 ||
      (bstride * 2) % 16 != 0)
    return fail(FM_E_INVALID, "TMA operand must be 16-byte aligned with 16-byte row/matrix strides");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(bstride * 2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                        swz == CU_TENSOR_MAP_SWIZZLE_NONE ? CU_TENSOR_MAP_L2_PROMOTION_NONE
                                                          : CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FM_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return FM_OK;
}

// Epilogue store map (32 x 32 boxes) of a destination, or *ok = false when
// its rows are not 16-byte aligned (the epilogue then stores directly).
int make_store_map(CUtensorMap* map, bool* ok, const void* base, long long batch, long long rows,
                   long long cols, long long ld, long long bstride) {
  const long long bs = batch == 1 ? round_up(rows * ld, 8) : bstride;
  *ok = (reinterpret_cast<uintptr_t>(base) & 15) == 0 && (ld * 2) % 16 == 0 && (bs * 2) % 16 == 0;
  if (!*ok) return FM_OK;
  return make_map(map, base, batch, rows, cols, ld, bstride, 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// GEMM kernel selection (fm_set_gemm_path): 0 = automatic, 1 = single-CTA
// 128x256 tiles, 2 = CTA-pair 256x256 tiles, 3 = persistent kernel over all
// iterations with 128x256 tiles, 4 = the same with 128x128 tiles.
std::atomic<int> g_gemm_path{0};

// Kernels this library has launched in the process (fm_launch_count).
std::atomic<unsigned long long> g_launches{0};
inline void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// CTA pairs of a 148-SM B200.  Split-K choices (and therefore workspace
// sizes) are made against this constant so fm_workspace_size needs no device.
constexpr int kRefPairs = 74;

struct GemmPlan {
  int tiles = 0;  // output tiles per matrix
  int split = 1;  // K-splits per tile
  int kbps = 0;   // K-blocks per split
};

struct NsPlan {
  bool pairs = false;
  GemmPlan g[3];  // X·Xᵀ, polynomial, B·X
  int tiles_m3 = 0, tiles_n3 = 0;
  long long split_slots = 0;  // max over GEMMs of batch*tiles*split (split > 1 only)
  long long counter_slots = 0;
};

// Split-K when a launch has fewer tiles than CTA pairs: at most 8 splits, at
// least 4 K-blocks (256 reduction elements) per split, no empty split.
GemmPlan plan_gemm(long long tiles, long long batch, int num_kb, bool pairs) {
  GemmPlan p;
  p.tiles = int(tiles);
  p.kbps = num_kb;
  const long long units = tiles * batch;
  if (!pairs || units >= kRefPairs) return p;
  int s = int(std::min<long long>(8, kRefPairs / units));
  s = std::min(s, std::max(1, num_kb / 4));
  if (s <= 1) return p;
  const int kbps = (num_kb + s - 1) / s;
  p.split = (num_kb + kbps - 1) / kbps;
  p.kbps = kbps;
  return p;
}

NsPlan plan_ns(long long batch, long long m, long long n, int path) {
  NsPlan P;
  P.pairs = path == 2 || (path == 0 && (m > 256 || batch > 1));
  const int kb1 = int((n + kBK - 1) / kBK), kb2 = int((m + kBK - 1) / kBK);
  const int bm = P.pairs ? kPairBM : kBM, bn = P.pairs ? kPairBN : kBN;
  const int t1 = P.pairs ? syrk_pair_tile_count(int(m)) : syrk_tile_count(int(m));
  P.tiles_m3 = int((m + bm - 1) / bm);
  P.tiles_n3 = int((n + bn - 1) / bn);
  P.g[0] = plan_gemm(t1, batch, kb1, P.pairs);
  P.g[1] = plan_gemm(t1, batch, kb2, P.pairs);
  P.g[2] = plan_gemm(static_cast<long long>(P.tiles_m3) * P.tiles_n3, batch, kb2, P.pairs);
  for (const GemmPlan& g : P.g) {
    if (g.split > 1) {
      P.split_slots = std::max(P.split_slots, batch * g.tiles * g.split);
      P.counter_slots = std::max(P.counter_slots, batch * g.tiles);
    }
  }
  return P;
}

// Workspace carve-up for `batch` m x n problems (m <= n after orientation).
struct Workspace {
  __nv_bfloat16* X[2];
  __nv_bfloat16* A;
  __nv_bfloat16* B;
  float* diag;
  float* partials;  // Frobenius-norm partials, kMaxPartials per matrix
  float* splitk;    // split-K fp32 partial tiles (128 KB per unit and CTA)
  int* counters;    // split-K arrival counters (two per tile: one per CTA)
  int* phase;       // persistent kernels: phase-completion counters (kFusedSlots),
                    // then at kRowdoneOffset the CTA-pair kernel's row-block counters
  long long ldx, ldm, xs, ms, dsz;  // row strides and per-matrix strides (elements)
  size_t counter_bytes;
  size_t bytes;
};

Workspace layout(long long batch, long long m, long long n, void* base) {
  Workspace w{};
  w.ldx = round_up(n, 8);
  w.ldm = round_up(m, 8);
  w.xs = round_up(m * w.ldx, 128);
  w.ms = round_up(m * w.ldm, 128);
  w.dsz = round_up(m, 64);
  // sized for the CTA-pair path, the larger of the two
  const NsPlan P = plan_ns(batch, m, n, 2);
  auto a256 = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t xb = a256(size_t(batch) * w.xs * 2), mb = a256(size_t(batch) * w.ms * 2);
  const size_t db = a256(size_t(batch) * w.dsz * 4), pb = a256(size_t(batch) * kMaxPartials * 4);
  const size_t sb = a256(size_t(P.split_slots) * 2 * kPartialFloats * 4);
  w.counter_bytes = a256(size_t(P.counter_slots) * 2 * 4);
  char* p = static_cast<char*>(base);
  size_t off = 0;
  w.X[0] = reinterpret_cast<__nv_bfloat16*>(p + off); off += xb;
  w.X[1] = reinterpret_cast<__nv_bfloat16*>(p + off); off += xb;
  w.A = reinterpret_cast<__nv_bfloat16*>(p + off); off += mb;
  w.B = reinterpret_cast<__nv_bfloat16*>(p + off); off += mb;
  w.diag = reinterpret_cast<float*>(p + off); off += db;
  w.partials = reinterpret_cast<float*>(p + off); off += pb;
  w.splitk = reinterpret_cast<float*>(p + off); off += sb;
  w.counters = reinterpret_cast<int*>(p + off); off += w.counter_bytes;
  w.phase = reinterpret_cast<int*>(p + off); off += kPhaseBytes;
  w.bytes = off;
  return w;
}

// Launch with programmatic stream serialization (PDL): the kernel may begin
// while the previous kernel on the stream drains; it waits (griddepcontrol)
// before touching global memory.  cluster2 adds a 2-CTA cluster dimension.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, bool cluster2, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster2) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e == cudaSuccess) note_launch();
  return e;
}

template <int MODE>
int launch_gemm(const DeviceState& ds, const CUtensorMap& ma, const CUtensorMap& mb,
                const CUtensorMap& mo, GemmArgs g, cudaStream_t st) {
  g.err = ds.err_word;
  if (g.num_tiles <= 0) return FM_OK;
  const int grid = std::min(g.num_tiles, ds.sm_count);
  const long long tm = timer_begin(MODE, st);
  FM_CUDA(launch_pdl(ns_gemm_kernel<MODE>, dim3(grid), dim3(kThreads), kSmemBytes, st, false, ma,
                     mb, mo, g));
  timer_end(tm, st);
  return FM_OK;
}

// CTA-pair launch: a cluster of 2 CTAs per 256x256 tile slot, one pair per
// two SMs, persistent over the work units.
template <int MODE>
int launch_gemm_pair(const DeviceState& ds, const CUtensorMap& ma, const CUtensorMap& mb,
                     const CUtensorMap& mo, GemmArgs g, cudaStream_t st) {
  g.err = ds.err_word;
  if (g.num_tiles <= 0) return FM_OK;
  const int pairs = std::min(g.num_tiles, ds.sm_count / 2);
  const long long tm = timer_begin(MODE, st);
  FM_CUDA(launch_pdl(ns_gemm_pair_kernel<MODE>, dim3(2 * pairs), dim3(kThreads), kPairSmemBytes, st,
                     true, ma, mb, mo, g));
  timer_end(tm, st);
  return FM_OK;
}

// Operands of one iteration for a batch: X (cur) -> X' (nxt).
struct IterIO {
  const __nv_bfloat16* cur;
  long long ldc, cur_bs;  // row / matrix stride of cur
  __nv_bfloat16* nxt;
  long long out_ld, out_bs;  // row / matrix stride of nxt (of X'ᵀ when transposed)
  int transpose_out;
};

template <int MODE>
int run_gemm(const DeviceState& ds, const NsPlan& P, const GemmPlan& gp, long long batch,
             const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, GemmArgs g,
             cudaStream_t st) {
  g.batch = int(batch);
  g.tiles = gp.tiles;
  g.split = gp.split;
  g.kb_per_split = gp.kbps;
  g.num_tiles = int(batch * gp.tiles * gp.split);
  if (P.pairs) return launch_gemm_pair<MODE>(ds, ma, mb, mo, g, st);
  g.num_tiles = gp.tiles;  // single-CTA kernel: batch == 1, split == 1
  return launch_gemm<MODE>(ds, ma, mb, mo, g, st);
}

int ns_iteration(const DeviceState& ds, const Workspace& w, const NsPlan& P, long long batch,
                 long long m, long long n, const IterIO& io, cudaStream_t st) {
  if (!P.pairs && batch > 1) {
    // single-CTA path (tests / tuning only): one matrix at a time
    for (long long b = 0; b < batch; ++b) {
      Workspace wb = w;
      wb.A = w.A + b * w.ms;
      wb.B = w.B + b * w.ms;
      wb.diag = w.diag + b * w.dsz;
      IterIO ib = io;
      ib.cur = io.cur + b * io.cur_bs;
      ib.nxt = io.nxt + b * io.out_bs;
      if (int rc = ns_iteration(ds, wb, P, 1, m, n, ib, st)) return rc;
    }
    return FM_OK;
  }
  CUtensorMap mx_k, mx_mn, ma, mbm, so_a, so_b, so_x;
  int rc;
  if ((rc = make_map(&mx_k, io.cur, batch, m, n, io.ldc, io.cur_bs, kBK, kBM))) return rc;
  if ((rc = make_map(&mx_mn, io.cur, batch, m, n, io.ldc, io.cur_bs, 64, kBK))) return rc;
  if ((rc = make_map(&ma, w.A, batch, m, m, w.ldm, w.ms, kBK, kBM))) return rc;
  if ((rc = make_map(&mbm, w.B, batch, m, m, w.ldm, w.ms, kBK, kBM))) return rc;
  bool ok_a, ok_b, ok_x;
  if ((rc = make_store_map(&so_a, &ok_a, w.A, batch, m, m, w.ldm, w.ms))) return rc;
  if ((rc = make_store_map(&so_b, &ok_b, w.B, batch, m, m, w.ldm, w.ms))) return rc;
  // X' (m x n), or X'ᵀ (n x m) when the last step writes a tall output
  if ((rc = make_store_map(&so_x, &ok_x, io.nxt, batch, io.transpose_out ? n : m,
                           io.transpose_out ? m : n, io.out_ld, io.out_bs)))
    return rc;

  GemmArgs base{};
  base.M = int(m);
  base.partial = w.splitk;
  base.counters = w.counters;
  base.tiles_m = P.tiles_m3;
  base.tiles_n = P.tiles_n3;

  // GEMM1: A = X·Xᵀ
  GemmArgs g1 = base;
  g1.N = int(m); g1.K = int(n);
  g1.out = w.A; g1.ld_out = w.ldm; g1.bs_out = w.ms;
  g1.tma_out = ok_a;
  if ((rc = run_gemm<kSyrk>(ds, P, P.g[0], batch, mx_k, mx_k, ok_a ? so_a : ma, g1, st))) return rc;

  // GEMM2: Boff = offdiag(c·A·A + b·A), diag = a + diag(c·A·A + b·A)
  GemmArgs g2 = base;
  g2.N = int(m); g2.K = int(m);
  g2.out = w.B; g2.ld_out = w.ldm; g2.bs_out = w.ms;
  g2.aux = w.A; g2.ld_aux = w.ldm; g2.bs_aux = w.ms;
  g2.diag = w.diag; g2.bs_diag = w.dsz;
  g2.tma_out = ok_b;
  if ((rc = run_gemm<kPoly>(ds, P, P.g[1], batch, ma, ma, ok_b ? so_b : ma, g2, st))) return rc;

  // GEMM3: X' = diag ⊙ X + Boff·X
  GemmArgs g3 = base;
  g3.N = int(n); g3.K = int(m);
  g3.out = io.nxt; g3.ld_out = io.out_ld; g3.bs_out = io.out_bs;
  g3.transpose_out = io.transpose_out;
  g3.aux = io.cur; g3.ld_aux = io.ldc; g3.bs_aux = io.cur_bs;
  g3.diag = w.diag; g3.bs_diag = w.dsz;
  g3.tma_out = ok_x;
  return run_gemm<kBX>(ds, P, P.g[2], batch, mbm, mx_mn, ok_x ? so_x : ma, g3, st);
}

int check_dims(long long rows, long long cols) {
  if (rows <= 0 || cols <= 0) return fail(FM_E_INVALID, "matrix must be non-empty, got %lld x %lld", rows, cols);
  // max side: the transposing prep kernel tiles the long side as 64-row blocks in grid.y
  if (std::min(rows, cols) > (1 << 20) || std::max(rows, cols) > 65535ll * 64)
    return fail(FM_E_INVALID, "matrix %lld x %lld too large", rows, cols);
  return FM_OK;
}

// Blocks of the norm / scale kernels: one per kPrepThreads * kFlatUnroll
// chunks, at most four per SM and kMaxPartials (the partials of one matrix).
int prep_grid(long long rows, long long cols, const DeviceState& ds) {
  const long long chunks = rows * ((cols + 7) / 8);
  const long long want = (chunks + kPrepThreads * kFlatUnroll - 1) / (kPrepThreads * kFlatUnroll);
  const long long cap = std::min<long long>(kMaxPartials, ds.sm_count * 4ll);
  return int(std::max<long long>(1, std::min(want, cap)));
}

// All `steps` iterations of a batch in one persistent launch (ns_fused_sm100.cuh):
// one CTA per SM, launched cooperatively so that every CTA is resident (the
// phase-completion waits rely on it), with programmatic stream serialization
// so its prologue overlaps the normalisation kernel.
// Maps and arguments shared by both persistent kernels (tile counts are set
// by the caller).
int fused_setup(const DeviceState& ds, const Workspace& w, long long batch, long long m,
                long long n, int steps, __nv_bfloat16* out, long long out_ld, long long out_bs,
                bool tall, FusedMaps& maps, FusedArgs& f) {
  int rc;
  for (int i = 0; i < 2; ++i) {
    if ((rc = make_map(&maps.xk[i], w.X[i], batch, m, n, w.ldx, w.xs, kBK, kBM))) return rc;
    if ((rc = make_map(&maps.xmn[i], w.X[i], batch, m, n, w.ldx, w.xs, 64, kBK))) return rc;
  }
  if ((rc = make_map(&maps.a, w.A, batch, m, m, w.ldm, w.ms, kBK, kBM))) return rc;
  if ((rc = make_map(&maps.b, w.B, batch, m, m, w.ldm, w.ms, kBK, kBM))) return rc;
  bool ok;
  if ((rc = make_store_map(&maps.so_a, &ok, w.A, batch, m, m, w.ldm, w.ms)) || !ok)
    return rc ? rc : fail(FM_E_INVALID, "workspace A not TMA-addressable");
  if ((rc = make_store_map(&maps.so_b, &ok, w.B, batch, m, m, w.ldm, w.ms)) || !ok)
    return rc ? rc : fail(FM_E_INVALID, "workspace B not TMA-addressable");
  for (int i = 0; i < 2; ++i)
    if ((rc = make_store_map(&maps.so_x[i], &ok, w.X[i], batch, m, n, w.ldx, w.xs)) || !ok)
      return rc ? rc : fail(FM_E_INVALID, "workspace X not TMA-addressable");
  bool ok_out;
  if ((rc = make_store_map(&maps.so_out, &ok_out, out, batch, tall ? n : m, tall ? m : n, out_ld,
                           out_bs)))
    return rc;
  if (!ok_out) maps.so_out = maps.so_x[0];  // unused: the last step stores directly
  f = FusedArgs{};
  f.M = int(m);
  f.N = int(n);
  f.batch = int(batch);
  f.steps = steps;
  f.X[0] = w.X[0];
  f.X[1] = w.X[1];
  f.ldx = w.ldx;
  f.xs = w.xs;
  f.A = w.A;
  f.B = w.B;
  f.ldm = w.ldm;
  f.ms = w.ms;
  f.diag = w.diag;
  f.dsz = w.dsz;
  f.out = out;
  f.out_ld = out_ld;
  f.out_bs = out_bs;
  f.transpose_out = tall ? 1 : 0;
  f.tma_out_final = ok_out ? 1 : 0;
  f.counters = w.phase;  // zeroed by the caller before the normalisation kernels
  f.rowdone = w.phase + kRowdoneOffset;
  f.err = ds.err_word;
  return FM_OK;
}

int fused_units(FusedArgs& f, long long batch, int steps) {
  const long long upi = batch * (2ll * f.t_syrk + static_cast<long long>(f.tiles_m3) * f.tiles_n3);
  if (upi * steps > (1ll << 30)) return fail(FM_E_INVALID, "too many work units for one launch");
  f.units_iter = int(upi);
  return FM_OK;
}

template <int BN>
int run_fused(const DeviceState& ds, const Workspace& w, long long batch, long long m, long long n,
              int steps, __nv_bfloat16* out, long long out_ld, long long out_bs, bool tall,
              cudaStream_t st) {
  FusedMaps maps;
  FusedArgs f;
  if (int rc = fused_setup(ds, w, batch, m, n, steps, out, out_ld, out_bs, tall, maps, f)) return rc;
  f.t_syrk = fused_syrk_tiles<BN>(int(m));
  f.tiles_m3 = int((m + kBM - 1) / kBM);
  f.tiles_n3 = int((n + BN - 1) / BN);
  if (int rc = fused_units(f, batch, steps)) return rc;
  const long long upi = f.units_iter;
  const int grid = int(std::min<long long>(ds.sm_count, upi * steps));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = FusedCfg<BN>::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const long long tm = timer_begin(4, st);
  FM_CUDA(cudaLaunchKernelEx(&cfg, ns_fused_kernel<BN>, maps, f));
  note_launch();
  timer_end(tm, st);
  return FM_OK;
}

// All iterations of a batch in one persistent launch on CTA-pair tiles
// (ns_fused2_sm100.cuh): 2-CTA clusters, one CTA per SM, cooperative.
int run_fused_pair(const DeviceState& ds, const Workspace& w, long long batch, long long m,
                   long long n, int steps, __nv_bfloat16* out, long long out_ld, long long out_bs,
                   bool tall, cudaStream_t st) {
  FusedMaps maps;
  FusedArgs f;
  if (int rc = fused_setup(ds, w, batch, m, n, steps, out, out_ld, out_bs, tall, maps, f)) return rc;
  const int T = int((m + kPairBM - 1) / kPairBM);
  if (T > kMaxPairRows) return fail(FM_E_INVALID, "matrix too large for the CTA-pair persistent kernel");
  f.t_syrk = T * (T + 1) / 2;
  f.tiles_m3 = T;
  f.tiles_n3 = int((n + kPairBN - 1) / kPairBN);
  if (int rc = fused_units(f, batch, steps)) return rc;
  const long long units = static_cast<long long>(f.units_iter) * steps;
  const int pairs = int(std::min<long long>(ds.sm_count / 2, units));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[3];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  attr[2].id = cudaLaunchAttributeClusterDimension;
  attr[2].val.clusterDim.x = 2;
  attr[2].val.clusterDim.y = 1;
  attr[2].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 3;
  const long long tm = timer_begin(4, st);
  FM_CUDA(cudaLaunchKernelEx(&cfg, ns_fused_pair_kernel, maps, f));
  note_launch();
  timer_end(tm, st);
  return FM_OK;
}

// Automatic choice of the persistent kernel (128 x 128 tiles): when one wave
// of SMs covers a whole SYRK phase, i.e. the batch's lower-triangle 128 x 128
// tiles fit on the SMs.  Then every phase is latency-bound (one tile per SM)
// and what the persistent kernel removes — a launch, grid drain and prologue
// per GEMM, and the CTA-pair path's split-K reductions — is most of the time.
// Larger problems keep one launch per GEMM on 256 x 256 CTA-pair tiles,
// whose mainloop is the more efficient one.
bool use_persistent(long long batch, long long m, const DeviceState& ds) {
  const long long mt = (m + kBM - 1) / kBM;
  return batch * (mt * (mt + 1) / 2) <= ds.sm_count;
}

// Automatic choice of the CTA-pair persistent kernel: a single matrix past
// the range above whose X (and A, B) stay in L2 — its B·X phase walks row
// blocks, which re-reads X once per row block.  Measured (power-capped, 30
// calls): 3072² 607 vs 636-678 µs, (3584, 4608) 1033-1040 vs 1098-1220 µs,
// 4096² 1235-1253 vs 1255 µs against one launch per GEMM; (4096, 6144) was
// 3% slower, so the bound stops below it.
bool use_persistent_pairs(long long batch, long long m, long long n) {
  return batch == 1 && m <= 4096 && m * n <= 4096ll * 4608ll;
}

// Full Newton-Schulz over a batch of same-shape matrices (batch = 1 for the
// single-matrix entry points).
// auto_persistent: whether the automatic path may pick the persistent kernel.
// Only the single-matrix entry points allow it.  The persistent kernel is a
// cooperative launch (all CTAs resident at once), so while other kernels hold
// SMs — e.g. NCCL collectives on another stream beside a sharded optimizer
// step, which uses the batched entry — it would wait for them to finish.
int ns_run(const void* G, int dtype, long long batch, long long rows, long long cols, long long ldg,
           long long bs_g, void* out, long long bs_out, int steps, void* workspace,
           uint64_t workspace_bytes, cudaStream_t st, bool auto_persistent) {
  if (!G || !out || !workspace) return fail(FM_E_INVALID, "null pointer argument");
  if (dtype < FM_DT_BF16 || dtype > FM_DT_F64) return fail(FM_E_INVALID, "unknown dtype %d", dtype);
  if (steps < 0) return fail(FM_E_INVALID, "steps must be >= 0, got %d", steps);
  if (batch < 1 || batch > 65535) return fail(FM_E_INVALID, "batch must be in [1, 65535], got %lld", batch);
  if (int rc = check_dims(rows, cols)) return rc;
  if (ldg < cols) return fail(FM_E_INVALID, "ldg %lld < cols %lld", ldg, cols);
  if (batch > 1 && (bs_g < rows * ldg || bs_out < rows * cols))
    return fail(FM_E_INVALID, "batch strides must not overlap matrices");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(FM_E_INVALID, "workspace must be 256-byte aligned");
  DeviceState* ds;
  if (int rc = device_state(&ds)) return rc;
  const bool tall = rows > cols;
  const long long m = tall ? cols : rows, n = tall ? rows : cols;
  Workspace w = layout(batch, m, n, workspace);
  if (workspace_bytes < w.bytes)
    return fail(FM_E_WORKSPACE, "workspace too small: need %zu bytes, got %llu", w.bytes,
                (unsigned long long)workspace_bytes);
  int path = g_gemm_path.load(std::memory_order_relaxed);
  if (path == 0 && auto_persistent) {
    if (use_persistent(batch, m, *ds)) {
      path = 4;
    } else if (use_persistent_pairs(batch, m, n)) {
      path = 5;
    }
  }
  const bool persistent = path == 3 || path == 4 || path == 5;
  const NsPlan P = plan_ns(batch, m, n, persistent ? 1 : path);
  auto* o = static_cast<__nv_bfloat16*>(out);

  const int pg = prep_grid(rows, cols, *ds);
  const long long tm = timer_begin(3, st);
  // Zero the counters a launch relies on before the normalisation kernels,
  // so the kernels that follow them keep their programmatic overlap.
  if (persistent && steps > 0) {
    FM_CUDA(cudaMemsetAsync(w.phase, 0, kPhaseBytes, st));
  } else if (P.split_slots > 0 && steps > 0) {
    FM_CUDA(cudaMemsetAsync(w.counters, 0, w.counter_bytes, st));
  }
  const long long bs_g_eff = batch > 1 ? bs_g : 0;
  FM_CUDA(launch_pdl(sumsq_kernel, dim3(pg, unsigned(batch)), dim3(kPrepThreads), 0, st, false,
                     G, dtype, rows, cols, ldg, bs_g_eff, w.partials));
  FM_CUDA(cudaGetLastError());
  if (steps == 0) {  // normalised input, original orientation
    FM_CUDA(launch_pdl(scale_kernel, dim3(pg, unsigned(batch)), dim3(kPrepThreads), 0, st, false,
                       G, dtype, rows, cols, ldg, bs_g_eff, (const float*)w.partials, pg, o,
                       (long long)cols, bs_out));
    FM_CUDA(cudaGetLastError());
    timer_end(tm, st);
    return FM_OK;
  }
  if (tall) {
    dim3 grid(unsigned((cols + kTC - 1) / kTC), unsigned((rows + kTR - 1) / kTR), unsigned(batch));
    FM_CUDA(launch_pdl(scale_transpose_kernel, grid, dim3(kPrepThreads), 0, st, false, G, dtype,
                       rows, cols, ldg, bs_g_eff, (const float*)w.partials, pg, w.X[0], w.ldx,
                       w.xs));
  } else {
    FM_CUDA(launch_pdl(scale_kernel, dim3(pg, unsigned(batch)), dim3(kPrepThreads), 0, st, false,
                       G, dtype, rows, cols, ldg, bs_g_eff, (const float*)w.partials, pg, w.X[0],
                       w.ldx, w.xs));
  }
  FM_CUDA(cudaGetLastError());
  timer_end(tm, st);
  if (persistent) {
    const long long out_ld = tall ? m : n;
    if (path == 5) return run_fused_pair(*ds, w, batch, m, n, steps, o, out_ld, bs_out, tall, st);
    return path == 3 ? run_fused<256>(*ds, w, batch, m, n, steps, o, out_ld, bs_out, tall, st)
                     : run_fused<128>(*ds, w, batch, m, n, steps, o, out_ld, bs_out, tall, st);
  }
  for (int i = 0; i < steps; ++i) {
    const bool last = i == steps - 1;
    IterIO io;
    io.cur = w.X[i & 1];
    io.ldc = w.ldx;
    io.cur_bs = w.xs;
    // The last step writes the caller's output directly: row-major m x n, or
    // its transpose (rows x cols = n x m) for tall inputs.
    io.nxt = last ? o : w.X[(i + 1) & 1];
    io.out_ld = last ? (tall ? m : n) : w.ldx;
    io.out_bs = last ? bs_out : w.xs;
    io.transpose_out = last && tall;
    if (int rc = ns_iteration(*ds, w, P, batch, m, n, io, st)) return rc;
  }
  return FM_OK;
}

}  // namespace
}  // namespace fm

using namespace fm;

extern "C" {

int fm_version(void) { return 100; }

const char* fm_last_error(void) { return t_err; }

int fm_workspace_size_batched(int64_t batch, int64_t rows, int64_t cols, uint64_t* bytes) {
  if (!bytes) return fail(FM_E_INVALID, "bytes is null");
  if (batch < 1 || batch > 65535) return fail(FM_E_INVALID, "batch must be in [1, 65535], got %lld", (long long)batch);
  if (int rc = check_dims(rows, cols)) return rc;
  const long long m = std::min(rows, cols), n = std::max(rows, cols);
  *bytes = layout(batch, m, n, nullptr).bytes;
  return FM_OK;
}

int fm_workspace_size(int64_t rows, int64_t cols, uint64_t* bytes) {
  return fm_workspace_size_batched(1, rows, cols, bytes);
}

int fm_fused_newton_schulz(const void* G, int dtype, int64_t rows, int64_t cols, int64_t ldg,
                           void* out, int steps, void* workspace, uint64_t workspace_bytes,
                           void* stream) {
  return ns_run(G, dtype, 1, rows, cols, ldg, 0, out, rows * cols, steps, workspace,
                workspace_bytes, static_cast<cudaStream_t>(stream), true);
}

int fm_fused_newton_schulz_batched(const void* G, int dtype, int64_t batch, int64_t rows,
                                   int64_t cols, int64_t ldg, int64_t batch_stride_g, void* out,
                                   int64_t batch_stride_out, int steps, void* workspace,
                                   uint64_t workspace_bytes, void* stream) {
  return ns_run(G, dtype, batch, rows, cols, ldg, batch_stride_g, out, batch_stride_out, steps,
                workspace, workspace_bytes, static_cast<cudaStream_t>(stream), false);
}

static int step_common(const void* X, int64_t m, int64_t n, int64_t ldx, void* X_new,
                       void* workspace, uint64_t workspace_bytes, void* stream, Workspace* wout) {
  if (!X || !X_new || !workspace) return fail(FM_E_INVALID, "null pointer argument");
  if (int rc = check_dims(m, n)) return rc;
  if (ldx < n) return fail(FM_E_INVALID, "ldx %lld < n %lld", (long long)ldx, (long long)n);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(FM_E_INVALID, "workspace must be 256-byte aligned");
  DeviceState* ds;
  if (int rc = device_state(&ds)) return rc;
  // The layout is sized for (min, max); a step on a tall X needs the m x m
  // intermediates, so size it as m x max(m, n).
  Workspace w = layout(1, m, std::max(m, n), workspace);
  if (workspace_bytes < w.bytes)
    return fail(FM_E_WORKSPACE, "workspace too small: need %zu bytes, got %llu", w.bytes,
                (unsigned long long)workspace_bytes);
  w.ldx = round_up(n, 8);
  w.xs = round_up(m * w.ldx, 128);
  const NsPlan P = plan_ns(1, m, n, g_gemm_path.load(std::memory_order_relaxed));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (P.split_slots > 0) FM_CUDA(cudaMemsetAsync(w.counters, 0, w.counter_bytes, st));
  IterIO io;
  io.cur = static_cast<const __nv_bfloat16*>(X);
  io.ldc = ldx;
  io.cur_bs = 0;
  if ((reinterpret_cast<uintptr_t>(X) & 15) != 0 || ldx % 8 != 0) {
    // Not TMA-addressable: copy into the workspace (no normalisation).
    const int pg = prep_grid(m, n, *ds);
    scale_kernel<<<dim3(pg, 1), kPrepThreads, 0, st>>>(X, FM_DT_BF16, m, n, ldx, 0, nullptr, 0,
                                                      w.X[0], w.ldx, w.xs);
    FM_CUDA(cudaGetLastError());
    note_launch();
    io.cur = w.X[0];
    io.ldc = w.ldx;
  }
  io.nxt = static_cast<__nv_bfloat16*>(X_new);
  io.out_ld = n;
  io.out_bs = m * n;
  io.transpose_out = 0;
  if (int rc = ns_iteration(*ds, w, P, 1, m, n, io, st)) return rc;
  *wout = w;
  return FM_OK;
}

int fm_newton_schulz_step(const void* X, int64_t m, int64_t n, int64_t ldx, void* X_new,
                          void* workspace, uint64_t workspace_bytes, void* stream) {
  Workspace w;
  return step_common(X, m, n, ldx, X_new, workspace, workspace_bytes, stream, &w);
}

int fm_ns_step_debug(const void* X, int64_t m, int64_t n, int64_t ldx, void* A, void* Boff,
                     float* diag, void* X_new, void* workspace, uint64_t workspace_bytes,
                     void* stream) {
  if (!A || !Boff || !diag) return fail(FM_E_INVALID, "null pointer argument");
  Workspace w;
  if (int rc = step_common(X, m, n, ldx, X_new, workspace, workspace_bytes, stream, &w)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  FM_CUDA(cudaMemcpy2DAsync(A, m * 2, w.A, w.ldm * 2, m * 2, m, cudaMemcpyDeviceToDevice, st));
  FM_CUDA(cudaMemcpy2DAsync(Boff, m * 2, w.B, w.ldm * 2, m * 2, m, cudaMemcpyDeviceToDevice, st));
  FM_CUDA(cudaMemcpyAsync(diag, w.diag, m * 4, cudaMemcpyDeviceToDevice, st));
  return FM_OK;
}

namespace {
int ew_grid(long long n, const DeviceState& ds) {
  const long long blocks = (n / 8 + kEwThreads - 1) / kEwThreads;
  return int(std::max<long long>(1, std::min<long long>(blocks, ds.sm_count * 8ll)));
}
}  // namespace

int fm_muon_momentum(void* buf, const void* grad, void* dir, int64_t n, int dtype, float momentum,
                     int nesterov, void* stream) {
  if (!buf || !grad || !dir) return fail(FM_E_INVALID, "null pointer argument");
  if (n < 0) return fail(FM_E_INVALID, "negative element count");
  if (n == 0) return FM_OK;
  DeviceState* ds;
  if (int rc = device_state(&ds)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* d = static_cast<__nv_bfloat16*>(dir);
  const int grid = ew_grid(n, *ds);
  switch (dtype) {
    case FM_DT_F32:
      muon_momentum_bf16dir_kernel<float><<<grid, kEwThreads, 0, st>>>(
          static_cast<float*>(buf), static_cast<const float*>(grad), d, n, momentum, nesterov);
      break;
    case FM_DT_BF16:
      muon_momentum_bf16dir_kernel<__nv_bfloat16><<<grid, kEwThreads, 0, st>>>(
          static_cast<__nv_bfloat16*>(buf), static_cast<const __nv_bfloat16*>(grad), d, n,
          momentum, nesterov);
      break;
    case FM_DT_F16:
      muon_momentum_bf16dir_kernel<__half><<<grid, kEwThreads, 0, st>>>(
          static_cast<__half*>(buf), static_cast<const __half*>(grad), d, n, momentum, nesterov);
      break;
    default:
      return fail(FM_E_INVALID, "fm_muon_momentum: unsupported dtype %d", dtype);
  }
  FM_CUDA(cudaGetLastError());
  note_launch();
  return FM_OK;
}

int fm_muon_apply(void* param, int dtype, const void* update, int64_t n, float decay, float alpha,
                  void* stream) {
  if (!param || !update) return fail(FM_E_INVALID, "null pointer argument");
  if (n < 0) return fail(FM_E_INVALID, "negative element count");
  if (n == 0) return FM_OK;
  DeviceState* ds;
  if (int rc = device_state(&ds)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* u = static_cast<const __nv_bfloat16*>(update);
  const int grid = ew_grid(n, *ds);
  switch (dtype) {
    case FM_DT_F32:
      muon_apply_kernel<float><<<grid, kEwThreads, 0, st>>>(static_cast<float*>(param), u, n, decay,
                                                            alpha);
      break;
    case FM_DT_BF16:
      muon_apply_kernel<__nv_bfloat16><<<grid, kEwThreads, 0, st>>>(
          static_cast<__nv_bfloat16*>(param), u, n, decay, alpha);
      break;
    case FM_DT_F16:
      muon_apply_kernel<__half><<<grid, kEwThreads, 0, st>>>(static_cast<__half*>(param), u, n,
                                                             decay, alpha);
      break;
    default:
      return fail(FM_E_INVALID, "fm_muon_apply: unsupported dtype %d", dtype);
  }
  FM_CUDA(cudaGetLastError());
  note_launch();
  return FM_OK;
}

int fm_set_gemm_path(int path) {
  if (path < 0 || path > 5) return fail(FM_E_INVALID, "gemm path must be in [0, 5], got %d", path);
  g_gemm_path.store(path);
  return FM_OK;
}

int fm_stage_timing(int enable) {
  t_timer.on = enable != 0;
  t_timer.used = 0;
  t_timer.marks.clear();
  return FM_OK;
}

int fm_launch_count(uint64_t* count) {
  if (!count) return fail(FM_E_INVALID, "null pointer argument");
  *count = g_launches.load(std::memory_order_relaxed);
  return FM_OK;
}

int fm_stage_times(float* ms, int* counts) {
  if (!ms || !counts) return fail(FM_E_INVALID, "null pointer argument");
  for (int i = 0; i < kStages4; ++i) {
    ms[i] = 0.f;
    counts[i] = 0;
  }
  StageTimer& T = t_timer;
  for (auto& mk : T.marks) {
    cudaEvent_t a = T.pool[mk.second], b = T.pool[mk.second + 1];
    FM_CUDA(cudaEventSynchronize(b));
    float t = 0.f;
    FM_CUDA(cudaEventElapsedTime(&t, a, b));
    ms[mk.first] += t;
    counts[mk.first] += 1;
  }
  T.used = 0;
  T.marks.clear();
  return FM_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of fm_fused_newton_schulz.
//
// Its scratch is this file-scope device array instead of a caller buffer.
// Every GPU that loads the library holds it until the process exits.  Host
// code cannot use the array's name as a device address, so the address is
// looked up with cudaGetSymbolAddress once per device, with that device
// current, on the first call made on that device.
static __device__ __align__(256) unsigned char g_static_scratch[FM_STATIC_SCRATCH_BYTES];

namespace {
std::atomic<void*> g_static_scratch_ptr[kMaxDevices];
std::mutex g_static_mu;

int static_scratch(void** out) {
  int dev = 0;
  FM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(FM_E_DEVICE, "device index %d out of range", dev);
  void* cached = g_static_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!cached) {
    std::lock_guard<std::mutex> lk(g_static_mu);
    cached = g_static_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (!cached) {
      FM_CUDA(cudaGetSymbolAddress(&cached, g_static_scratch));
      if (!cached) return fail(FM_E_CUDA, "cudaGetSymbolAddress returned a null scratch address");
      g_static_scratch_ptr[dev].store(cached, std::memory_order_release);
    }
  }
  *out = cached;
  return FM_OK;
}
}  // namespace

int fm_fused_newton_schulz_noalloc(const void* G, int dtype, int64_t rows, int64_t cols,
                                   int64_t ldg, void* out, int steps, void* stream) {
  if (rows > 0 && cols > 0) {
    uint64_t need = 0;
    if (int rc = fm_workspace_size(rows, cols, &need)) return rc;
    if (need > FM_STATIC_SCRATCH_BYTES)
      return fail(FM_E_WORKSPACE,
                  "fm_fused_newton_schulz_noalloc: a %lld x %lld matrix needs %llu scratch bytes, "
                  "more than the library's fixed %llu-byte device scratch; use "
                  "fm_fused_newton_schulz with a caller-allocated workspace",
                  (long long)rows, (long long)cols, (unsigned long long)need,
                  (unsigned long long)FM_STATIC_SCRATCH_BYTES);
  }
  void* scratch = nullptr;
  if (int rc = static_scratch(&scratch)) return rc;
  // Nothing in the scratch has to start at zero: every byte a call reads
  // (norm partials, X buffers, A, B, diagonal) is written earlier in the same call.
  return fm_fused_newton_schulz(G, dtype, rows, cols, ldg, out, steps, scratch,
                                FM_STATIC_SCRATCH_BYTES, stream);
}

int fm_selftest_wait_timeout(void* stream) {
  DeviceState* ds;
  if (int rc = device_state(&ds)) return rc;
  // One single-CTA GEMM launch over a tiny valid operand whose producer is
  // told to issue nothing: the MMA warp's wait on the first stage has nothing
  // to wait for, gives up after its budget, records kErrWaitFull and the CTA
  // frees its TMEM and exits.  No memory is written; nothing is allocated
  // beyond a 2 KB scratch operand.
  static __nv_bfloat16* operand[kMaxDevices] = {};
  int dev = 0;
  FM_CUDA(cudaGetDevice(&dev));
  if (!operand[dev]) FM_CUDA(cudaMalloc(&operand[dev], 128 * 8 * sizeof(__nv_bfloat16)));
  CUtensorMap map;
  if (int rc = make_map(&map, operand[dev], 1, 128, 8, 8, 0, kBK, kBM)) return rc;
  GemmArgs g{};
  g.M = 128; g.N = 128; g.K = 8;
  g.num_tiles = 1;
  g.out = operand[dev]; g.ld_out = 8;
  g.batch = 1; g.tiles = 1; g.split = 1; g.kb_per_split = 1;
  g.starve = 1;
  return launch_gemm<kSyrk>(*ds, map, map, map, g, static_cast<cudaStream_t>(stream));
}

int fm_device_error(uint32_t* code) {
  if (!code) return fail(FM_E_INVALID, "code is null");
  DeviceState* ds;
  if (int rc = device_state(&ds)) return rc;
  FM_CUDA(cudaDeviceSynchronize());
  unsigned v = 0;
  FM_CUDA(cudaMemcpy(&v, ds->err_word, sizeof(v), cudaMemcpyDeviceToHost));
  const unsigned zero = 0;
  FM_CUDA(cudaMemcpy(ds->err_word, &zero, sizeof(zero), cudaMemcpyHostToDevice));
  *code = v;
  return FM_OK;
}

}  // extern "C"

#ifdef FM_TRACE
// Development only: copy the CTA-pair timeline (128 x 40 u64) to host memory.
extern "C" int fm_trace_read(void* host) {
  FM_CUDA(cudaDeviceSynchronize());
  FM_CUDA(cudaMemcpyFromSymbol(host, fm::g_fm_trace, sizeof(fm::g_fm_trace)));
  return FM_OK;
}
// Development only: the persistent kernel's timeline (160 x 64 x 4 u64).
extern "C" int fm_fused_trace_read(void* host) {
  FM_CUDA(cudaDeviceSynchronize());
  FM_CUDA(cudaMemcpyFromSymbol(host, fm::g_fused_trace, sizeof(fm::g_fused_trace)));
  return FM_OK;
}
#endif
