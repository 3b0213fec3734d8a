/*
 * fused_muon.h — C ABI of the B200 (sm_100a) Newton-Schulz engine.
 *
 * Plain pointers, sizes and a CUDA stream handle (passed as void*); no torch
 * or C++ types cross this boundary.  Every call is asynchronous on `stream`
 * and returns 0 on success or a negative FM_E* code; fm_last_error() gives a
 * message for the calling thread's last failure.  Device pointers must be
 * on the current CUDA device.
 *
 * Each entry point names the reference interface it replaces
 * (StarrickLiu/fused-muon).
 */
#ifndef FUSED_MUON_H_
#define FUSED_MUON_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define FM_OK 0
#define FM_E_INVALID (-1)   /* bad argument (shape, pointer, dtype, size) */
#define FM_E_WORKSPACE (-2) /* workspace smaller than fm_workspace_size() */
#define FM_E_CUDA (-3)      /* CUDA runtime / driver error */
#define FM_E_DEVICE (-4)    /* unsupported device (needs sm_100) */

/* Input element types accepted by fm_fused_newton_schulz (output is bf16). */
#define FM_DT_BF16 0
#define FM_DT_F16 1
#define FM_DT_F32 2
#define FM_DT_F64 3

/* Library version, e.g. 100 for 0.1.0. */
int fm_version(void);

/* Message for the calling thread's most recent failed call ("" if none). */
const char* fm_last_error(void);

/*
 * Workspace bytes needed by fm_fused_newton_schulz / fm_newton_schulz_step for
 * a rows x cols matrix (either orientation).
 * Replaces: csrc/ns_gemm.cu:37-52 newton_schulz_workspace_size(m, n) and
 * csrc/torch_binding.cu:16-18 query_workspace_size (exported as
 * _C.workspace_size, torch_binding.cu:132-134).
 */
int fm_workspace_size(int64_t rows, int64_t cols, uint64_t* bytes);

/*
 * Full Newton-Schulz orthogonalisation: out = NS_steps(G) in bf16.
 * G: rows x cols, row stride ldg (elements), element type `dtype`.
 * out: rows x cols bf16, contiguous.  Tall inputs (rows > cols) are handled
 * by working on Gᵀ and writing the result back transposed.
 * workspace: device buffer of at least fm_workspace_size(rows, cols) bytes,
 * 256-byte aligned.
 * Replaces: csrc/torch_binding.cu:58-123 fused_newton_schulz (pybind
 * _C.fused_newton_schulz) and the Python front muon_fused/ns_step.py:85-123.
 */
int fm_fused_newton_schulz(const void* G, int dtype, int64_t rows, int64_t cols, int64_t ldg,
                           void* out, int steps, void* workspace, uint64_t workspace_bytes,
                           void* stream);

/*
 * Batched form: `batch` same-shape matrices G_b = G + b * batch_stride_g
 * (elements), each orthogonalised independently into
 * out + b * batch_stride_out (bf16, rows x cols contiguous per matrix).  One
 * set of GEMM launches covers the whole batch, so small matrices fill the GPU.
 * workspace: at least fm_workspace_size_batched(batch, rows, cols) bytes.
 * Replaces: the reference's per-matrix loop of fused_newton_schulz calls
 * inside FusedMuon.step (muon_fused/optimizer.py:128-163).
 */
int fm_workspace_size_batched(int64_t batch, int64_t rows, int64_t cols, uint64_t* bytes);
int fm_fused_newton_schulz_batched(const void* G, int dtype, int64_t batch, int64_t rows,
                                   int64_t cols, int64_t ldg, int64_t batch_stride_g, void* out,
                                   int64_t batch_stride_out, int steps, void* workspace,
                                   uint64_t workspace_bytes, void* stream);

/*
 * One Newton-Schulz iteration on an already normalised bf16 matrix:
 * X_new = (a·I + b·A + c·A²)·X with A = X·Xᵀ.  X: m x n bf16 with row stride
 * ldx; X_new: m x n bf16, contiguous.  No transpose is applied.
 * Replaces: csrc/ns_gemm.h:20-25 xcompute::newton_schulz_step and
 * csrc/torch_binding.cu:22-54 ns_step (pybind _C.newton_schulz_step).
 */
int fm_newton_schulz_step(const void* X, int64_t m, int64_t n, int64_t ldx, void* X_new,
                          void* workspace, uint64_t workspace_bytes, void* stream);

/*
 * Debug form of one iteration that also returns the intermediates:
 * A = X·Xᵀ (m x m bf16), Boff = off-diagonal part of b·A + c·A² (m x m bf16,
 * zero diagonal), diag = a + diagonal of b·A + c·A² (m floats), X_new as in
 * fm_newton_schulz_step.  All outputs contiguous.
 * Replaces: nothing exported by the reference; it exposes the products of the
 * reference's GEMM1/GEMM2 (csrc/ns_gemm.cu:94-118) for symmetry tests.
 */
int fm_ns_step_debug(const void* X, int64_t m, int64_t n, int64_t ldx, void* A, void* Boff,
                     float* diag, void* X_new, void* workspace, uint64_t workspace_bytes,
                     void* stream);

/*
 * Reads and clears the device-side error word of the current device
 * (synchronises the device).  *code is 0 when no kernel reported a timed-out
 * pipeline wait since the last call.
 * Replaces: nothing; the reference checks no kernel status
 * (csrc/syrk_64.cu:45-49, csrc/ns_gemm.cu:97,127).
 */
int fm_device_error(uint32_t* code);

/*
 * Failure-detection self-test: launches one GEMM whose loads are withheld,
 * so its pipeline wait runs out (after about two seconds) and the kernel
 * ends, reporting code 1 ("MMA warp timed out waiting for a stage") through
 * fm_device_error().  The context stays usable.  Nothing on the GPU faults,
 * traps or hangs.
 * Replaces: nothing; the reference has no failure detection beyond a silent
 * Python fallback (muon_fused/ns_step.py:117-120).
 */
int fm_selftest_wait_timeout(void* stream);

/*
 * Allocation-free form of fm_fused_newton_schulz, for callers that cannot
 * call cudaMalloc: code running inside a fixed memory budget (a host
 * framework that owns all device memory through its own pool), or code on a
 * path where an allocation could block or fail mid-step.  The caller passes
 * G and out as for fm_fused_newton_schulz; the scratch is a fixed device
 * array of FM_STATIC_SCRATCH_BYTES inside the library, which every GPU that
 * loads the library holds until the process exits.
 * - Limit: matrices whose fm_workspace_size() exceeds FM_STATIC_SCRATCH_BYTES
 *   are rejected with FM_E_WORKSPACE (e.g. 2048 x 2048 or 1024 x 4096
 *   fit; 4096 x 4096 does not).
 * - The first call on each device looks up the array's device address; make
 *   that first call before capturing the stream into a CUDA graph.
 * - All calls on a device share the one array, which keeps the last call's
 *   contents: calls that overlap on the GPU (other streams, other threads)
 *   race and corrupt each other.  Serialise them on one stream.
 * - Allocates nothing: no cudaMalloc/cudaFree or allocating library call.
 * Replaces: nothing; the reference has no counterpart (its binding always
 * allocates a workspace when none is passed, csrc/torch_binding.cu:93-103).
 */
#define FM_STATIC_SCRATCH_BYTES (64ull << 20)
int fm_fused_newton_schulz_noalloc(const void* G, int dtype, int64_t rows, int64_t cols,
                                   int64_t ldg, void* out, int steps, void* stream);

/*
 * Muon momentum in one pass over n elements of dtype FM_DT_F32 / BF16 / F16:
 *   buf = round(round(buf * momentum) + grad)
 *   dir = bf16(round(grad + momentum * buf))   if nesterov
 *   dir = bf16(buf)                            otherwise
 * where round() is rounding to the buffer's dtype after each torch op of the
 * reference, so buf is bit-identical to the reference's; dir is the bf16
 * Newton-Schulz input (the reference casts to bf16 inside NS, ns_step.py:40).
 * Replaces: muon_fused/optimizer.py:139-149 (buf.mul_(mu).add_(g);
 * g.add(buf, alpha=mu)).
 */
int fm_muon_momentum(void* buf, const void* grad, void* dir, int64_t n, int dtype, float momentum,
                     int nesterov, void* stream);

/*
 * Decoupled weight decay + update in one pass: for n elements of the
 * parameter (dtype FM_DT_F32 / BF16 / F16) and the bf16 update u,
 *   p = round(round(p * decay) + alpha * u)
 * with decay = 1 - lr*wd and alpha = -lr * 0.2 * sqrt(max(A, B)).
 * Replaces: muon_fused/optimizer.py:157-163 (p.data.mul_(1 - lr*wd);
 * p.data.add_(u, alpha=-adjusted_lr)).
 */
int fm_muon_apply(void* param, int dtype, const void* update, int64_t n, float decay, float alpha,
                  void* stream);

/*
 * GEMM kernel selection for all later calls in the process:
 * 0 = automatic: a single-matrix call (fm_fused_newton_schulz, the
 *     allocation-free form) whose lower-triangle 128x128 tiles fit on the SMs
 *     runs the persistent kernel (path 4, one cooperative launch for all
 *     iterations); a larger single matrix with m <= 4096 and m*n <=
 *     4096*4608 the CTA-pair persistent kernel (path 5); everything else,
 *     and every batched call, one launch per GEMM on CTA-pair tiles,
 * 1 = one launch per GEMM with single-CTA 128x256 tiles,
 * 2 = one launch per GEMM with CTA-pair 256x256 tiles, 3 = one persistent
 * launch for all iterations with 128x256 tiles, 4 = the same with 128x128
 * tiles, 5 = the same with CTA-pair 256x256 tiles, where the next iteration's
 * X·Xᵀ tiles start on finished row blocks of X'.  All produce the same
 * arithmetic (up to fp32 summation order where a path splits K); the switch
 * exists for tests and tuning.
 * Replaces: the reference's compile-time tile dispatch, csrc/ns_gemm.cu:68-92.
 */
int fm_set_gemm_path(int path);

/*
 * Benchmark instrumentation.  fm_stage_timing(1) makes every later launch of
 * the calling thread record a CUDA event pair around itself on its stream
 * (fm_stage_timing(0) stops it; either call discards pending pairs).
 * fm_stage_times() waits for the recorded events and returns, per stage, the
 * summed milliseconds and the launch count since the last read:
 * [0] GEMM1 A = X·Xᵀ, [1] GEMM2 polynomial, [2] GEMM3 X' = B·X, [3] norm/scale,
 * [4] the persistent kernel that runs all iterations in one launch.
 * Replaces: nothing; the reference has no instrumentation
 * (its timing lives in benchmarks/bench_ns_step.py:53-81).
 */
int fm_stage_timing(int enable);
int fm_stage_times(float* ms, int* counts);

/*
 * Number of kernels this library has launched in the calling process since it
 * was loaded (all devices, all threads); a benchmark reads it before and after
 * its timed region.
 * Replaces: nothing (benchmark instrumentation).
 */
int fm_launch_count(uint64_t* count);

#ifdef FM_TRACE
/*
 * Development builds only (compiled with -DFM_TRACE; the shipped library does
 * not export these).  Copy the kernels' %globaltimer timelines to host memory
 * after synchronising the device: fm_trace_read the CTA-pair GEMMs' (3 modes x
 * 128 pairs x 40 u64), fm_fused_trace_read the persistent kernel's
 * (160 CTAs x 64 units x 4 u64).
 * Replaces: nothing (instrumentation).
 */
int fm_trace_read(void* host);
int fm_fused_trace_read(void* host);
#endif

#ifdef __cplusplus
}
#endif

#endif /* FUSED_MUON_H_ */
