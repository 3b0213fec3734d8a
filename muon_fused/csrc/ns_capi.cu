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

struct DeviceState {
  bool ready = false;
  int sm_count = 0;
  unsigned* err_word = nullptr;
};
DeviceState g_dev[kMaxDevices];
std::mutex g_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

inline long long round_up(long long x, long long a) { return (x + a - 1) / a * a; }

// Optional per-stage timing for benchmarks (fm_stage_timing / fm_stage_times):
// when enabled, each kernel launch of this thread is bracketed by CUDA events
// on its stream; the pairs are resolved and summed per stage on request.
constexpr int kStages4 = 4;  // 0 GEMM1 (X·Xᵀ), 1 GEMM2 (poly), 2 GEMM3 (B·X), 3 prep kernels
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
  if (!s.ready) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!s.ready) {
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
      FM_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&s.err_word), g_device_error));
      if (!g_encode) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        FM_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn)
          return fail(FM_E_CUDA, "cuTensorMapEncodeTiled entry point not found");
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      }
      s.ready = true;
    }
  }
  *out = &s;
  return FM_OK;
}

// 2-D bf16 tensor map over a rows x cols row-major matrix with row stride ld
// (elements), box = box_cols (inner) x box_rows, 128-byte swizzle, zero fill
// out of bounds.
int make_map(CUtensorMap* map, const void* base, long long rows, long long cols, long long ld,
             int box_cols, int box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * 2) % 16 != 0)
    return fail(FM_E_INVALID, "TMA operand must be 16-byte aligned with 16-byte row stride");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FM_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return FM_OK;
}

// Workspace carve-up for an m x n problem (m <= n after orientation).
struct Workspace {
  __nv_bfloat16* X[2];
  __nv_bfloat16* A;
  __nv_bfloat16* B;
  float* diag;
  float* partials;
  long long ldx, ldm;
  size_t bytes;
};

Workspace layout(long long m, long long n, void* base) {
  Workspace w{};
  w.ldx = round_up(n, 8);
  w.ldm = round_up(m, 8);
  auto a256 = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t xb = a256(size_t(m) * w.ldx * 2), mb = a256(size_t(m) * w.ldm * 2);
  const size_t db = a256(size_t(m) * 4), pb = a256(kMaxPartials * 4);
  char* p = static_cast<char*>(base);
  size_t off = 0;
  w.X[0] = reinterpret_cast<__nv_bfloat16*>(p + off); off += xb;
  w.X[1] = reinterpret_cast<__nv_bfloat16*>(p + off); off += xb;
  w.A = reinterpret_cast<__nv_bfloat16*>(p + off); off += mb;
  w.B = reinterpret_cast<__nv_bfloat16*>(p + off); off += mb;
  w.diag = reinterpret_cast<float*>(p + off); off += db;
  w.partials = reinterpret_cast<float*>(p + off); off += pb;
  w.bytes = off;
  return w;
}

// GEMM kernel selection (fm_set_gemm_path): 0 = automatic, 1 = single-CTA
// 128x256 tiles, 2 = CTA-pair 256x256 tiles.  Automatic uses CTA pairs once
// the matrix spans more than one 256-row block.
std::atomic<int> g_gemm_path{0};

bool use_pairs(long long m) {
  const int p = g_gemm_path.load(std::memory_order_relaxed);
  if (p == 1) return false;
  if (p == 2) return true;
  return m > 256;
}

template <int MODE>
int launch_gemm(const DeviceState& ds, const CUtensorMap& ma, const CUtensorMap& mb, GemmArgs g,
                cudaStream_t st) {
  g.err = ds.err_word;
  if (g.num_tiles <= 0) return FM_OK;
  const int grid = std::min(g.num_tiles, ds.sm_count);
  const long long tm = timer_begin(MODE, st);
  ns_gemm_kernel<MODE><<<grid, kThreads, kSmemBytes, st>>>(ma, mb, g);
  FM_CUDA(cudaGetLastError());
  timer_end(tm, st);
  return FM_OK;
}

// CTA-pair launch: a cluster of 2 CTAs per 256x256 tile slot, one pair per
// two SMs, persistent over the tiles.
template <int MODE>
int launch_gemm_pair(const DeviceState& ds, const CUtensorMap& ma, const CUtensorMap& mb,
                     GemmArgs g, cudaStream_t st) {
  g.err = ds.err_word;
  if (g.num_tiles <= 0) return FM_OK;
  const int pairs = std::min(g.num_tiles, ds.sm_count / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const long long tm = timer_begin(MODE, st);
  FM_CUDA(cudaLaunchKernelEx(&cfg, ns_gemm_pair_kernel<MODE>, ma, mb, g));
  timer_end(tm, st);
  return FM_OK;
}

// One iteration: cur (m x n, ld w.ldx or given) -> nxt.
// out_ld / transpose_out describe how X' is stored.
int ns_iteration(const DeviceState& ds, const Workspace& w, const __nv_bfloat16* cur, long long ldc,
                 long long m, long long n, __nv_bfloat16* nxt, long long out_ld, int transpose_out,
                 cudaStream_t st) {
  CUtensorMap mx_k, mx_mn, ma, mbm;
  int rc;
  if ((rc = make_map(&mx_k, cur, m, n, ldc, kBK, kBM))) return rc;
  if ((rc = make_map(&mx_mn, cur, m, n, ldc, 64, kBK))) return rc;
  if ((rc = make_map(&ma, w.A, m, m, w.ldm, kBK, kBM))) return rc;
  if ((rc = make_map(&mbm, w.B, m, m, w.ldm, kBK, kBM))) return rc;
  const bool pairs = use_pairs(m);

  // GEMM1: A = X·Xᵀ
  GemmArgs g1{};
  g1.M = int(m); g1.N = int(m); g1.K = int(n);
  g1.out = w.A; g1.ld_out = w.ldm;
  if (pairs) {
    g1.num_tiles = syrk_pair_tile_count(int(m));
    rc = launch_gemm_pair<kSyrk>(ds, mx_k, mx_k, g1, st);
  } else {
    g1.num_tiles = syrk_tile_count(int(m));
    rc = launch_gemm<kSyrk>(ds, mx_k, mx_k, g1, st);
  }
  if (rc) return rc;

  // GEMM2: Boff = offdiag(c·A·A + b·A), diag = a + diag(c·A·A + b·A)
  GemmArgs g2{};
  g2.M = int(m); g2.N = int(m); g2.K = int(m);
  g2.out = w.B; g2.ld_out = w.ldm;
  g2.aux = w.A; g2.ld_aux = w.ldm;
  g2.diag = w.diag;
  if (pairs) {
    g2.num_tiles = syrk_pair_tile_count(int(m));
    rc = launch_gemm_pair<kPoly>(ds, ma, ma, g2, st);
  } else {
    g2.num_tiles = syrk_tile_count(int(m));
    rc = launch_gemm<kPoly>(ds, ma, ma, g2, st);
  }
  if (rc) return rc;

  // GEMM3: X' = diag ⊙ X + Boff·X
  GemmArgs g3{};
  g3.M = int(m); g3.N = int(n); g3.K = int(m);
  g3.out = nxt; g3.ld_out = out_ld; g3.transpose_out = transpose_out;
  g3.aux = cur; g3.ld_aux = ldc;
  g3.diag = w.diag;
  const int bm = pairs ? kPairBM : kBM, bn = pairs ? kPairBN : kBN;
  g3.tiles_n = int((n + bn - 1) / bn);
  g3.tiles_m = int((m + bm - 1) / bm);
  g3.num_tiles = g3.tiles_m * g3.tiles_n;
  return pairs ? launch_gemm_pair<kBX>(ds, mbm, mx_mn, g3, st)
               : launch_gemm<kBX>(ds, mbm, mx_mn, g3, st);
}

int check_dims(long long rows, long long cols) {
  if (rows <= 0 || cols <= 0) return fail(FM_E_INVALID, "matrix must be non-empty, got %lld x %lld", rows, cols);
  // max side: the transposing prep kernel tiles the long side as 64-row blocks in grid.y
  if (std::min(rows, cols) > (1 << 20) || std::max(rows, cols) > 65535ll * 64)
    return fail(FM_E_INVALID, "matrix %lld x %lld too large", rows, cols);
  return FM_OK;
}

int prep_grid(long long rows, const DeviceState& ds) {
  return int(std::min<long long>(std::min<long long>(rows, kMaxPartials), ds.sm_count * 4));
}

}  // namespace
}  // namespace fm

using namespace fm;

extern "C" {

int fm_version(void) { return 100; }

const char* fm_last_error(void) { return t_err; }

int fm_workspace_size(int64_t rows, int64_t cols, uint64_t* bytes) {
  if (!bytes) return fail(FM_E_INVALID, "bytes is null");
  if (int rc = check_dims(rows, cols)) return rc;
  const long long m = std::min(rows, cols), n = std::max(rows, cols);
  *bytes = layout(m, n, nullptr).bytes;
  return FM_OK;
}

int fm_fused_newton_schulz(const void* G, int dtype, int64_t rows, int64_t cols, int64_t ldg,
                           void* out, int steps, void* workspace, uint64_t workspace_bytes,
                           void* stream) {
  if (!G || !out || !workspace) return fail(FM_E_INVALID, "null pointer argument");
  if (dtype < FM_DT_BF16 || dtype > FM_DT_F64) return fail(FM_E_INVALID, "unknown dtype %d", dtype);
  if (steps < 0) return fail(FM_E_INVALID, "steps must be >= 0, got %d", steps);
  if (int rc = check_dims(rows, cols)) return rc;
  if (ldg < cols) return fail(FM_E_INVALID, "ldg %lld < cols %lld", (long long)ldg, (long long)cols);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(FM_E_INVALID, "workspace must be 256-byte aligned");
  DeviceState* ds;
  if (int rc = device_state(&ds)) return rc;
  const bool tall = rows > cols;
  const long long m = tall ? cols : rows, n = tall ? rows : cols;
  Workspace w = layout(m, n, workspace);
  if (workspace_bytes < w.bytes)
    return fail(FM_E_WORKSPACE, "workspace too small: need %zu bytes, got %llu", w.bytes,
                (unsigned long long)workspace_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* o = static_cast<__nv_bfloat16*>(out);

  const int pg = prep_grid(rows, *ds);
  const long long tm = timer_begin(3, st);
  sumsq_kernel<<<pg, kPrepThreads, 0, st>>>(G, dtype, rows, cols, ldg, w.partials);
  FM_CUDA(cudaGetLastError());
  if (steps == 0) {  // normalised input, original orientation
    scale_kernel<<<pg, kPrepThreads, 0, st>>>(G, dtype, rows, cols, ldg, w.partials, pg, o, cols);
    FM_CUDA(cudaGetLastError());
    return FM_OK;
  }
  if (tall) {
    dim3 grid(unsigned((cols + kTT - 1) / kTT), unsigned((rows + kTT - 1) / kTT));
    scale_transpose_kernel<<<grid, kPrepThreads, 0, st>>>(G, dtype, rows, cols, ldg, w.partials,
                                                          pg, w.X[0], w.ldx);
  } else {
    scale_kernel<<<pg, kPrepThreads, 0, st>>>(G, dtype, rows, cols, ldg, w.partials, pg, w.X[0],
                                              w.ldx);
  }
  FM_CUDA(cudaGetLastError());
  timer_end(tm, st);
  for (int i = 0; i < steps; ++i) {
    const __nv_bfloat16* cur = w.X[i & 1];
    const bool last = i == steps - 1;
    __nv_bfloat16* nxt = last ? o : w.X[(i + 1) & 1];
    // Last step writes the caller's output directly: row-major m x n, or its
    // transpose (rows x cols = n x m) for tall inputs.
    const long long out_ld = last ? (tall ? m : n) : w.ldx;
    if (int rc = ns_iteration(*ds, w, cur, w.ldx, m, n, nxt, out_ld, last && tall, st)) return rc;
  }
  return FM_OK;
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
  Workspace w = layout(m, std::max(m, n), workspace);
  if (workspace_bytes < w.bytes)
    return fail(FM_E_WORKSPACE, "workspace too small: need %zu bytes, got %llu", w.bytes,
                (unsigned long long)workspace_bytes);
  w.ldx = round_up(n, 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const __nv_bfloat16* cur = static_cast<const __nv_bfloat16*>(X);
  long long ldc = ldx;
  if ((reinterpret_cast<uintptr_t>(X) & 15) != 0 || ldx % 8 != 0) {
    // Not TMA-addressable: copy into the workspace (no normalisation).
    const int pg = prep_grid(m, *ds);
    scale_kernel<<<pg, kPrepThreads, 0, st>>>(X, FM_DT_BF16, m, n, ldx, nullptr, 0, w.X[0], w.ldx);
    FM_CUDA(cudaGetLastError());
    cur = w.X[0];
    ldc = w.ldx;
  }
  if (int rc = ns_iteration(*ds, w, cur, ldc, m, n, static_cast<__nv_bfloat16*>(X_new), n, 0, st))
    return rc;
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

int fm_set_gemm_path(int path) {
  if (path < 0 || path > 2) return fail(FM_E_INVALID, "gemm path must be 0, 1 or 2, got %d", path);
  g_gemm_path.store(path);
  return FM_OK;
}

int fm_stage_timing(int enable) {
  t_timer.on = enable != 0;
  t_timer.used = 0;
  t_timer.marks.clear();
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
void* g_static_scratch_ptr[kMaxDevices];
std::mutex g_static_mu;

int static_scratch(void** out) {
  int dev = 0;
  FM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(FM_E_DEVICE, "device index %d out of range", dev);
  if (!g_static_scratch_ptr[dev]) {
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_scratch_ptr[dev]) {
      void* p = nullptr;
      FM_CUDA(cudaGetSymbolAddress(&p, g_static_scratch));
      if (!p) return fail(FM_E_CUDA, "cudaGetSymbolAddress returned a null scratch address");
      g_static_scratch_ptr[dev] = p;
    }
  }
  *out = g_static_scratch_ptr[dev];
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
