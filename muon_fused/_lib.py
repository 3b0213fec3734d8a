"""ctypes binding of the C ABI in ``include/fused_muon.h``.

The native library is mandatory: there is no CPU or PyTorch fallback.  If the
library is missing or cannot be loaded, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfused_muon.so")

# Status codes and dtype codes mirrored from include/fused_muon.h.
FM_OK = 0
FM_E_INVALID = -1
FM_E_WORKSPACE = -2
FM_E_CUDA = -3
FM_E_DEVICE = -4
FM_DT_BF16, FM_DT_F16, FM_DT_F32, FM_DT_F64 = 0, 1, 2, 3

# Every symbol the header declares, with its ctypes signature.
_c_int, _i64, _u64, _vp = ctypes.c_int, ctypes.c_int64, ctypes.c_uint64, ctypes.c_void_p
SIGNATURES = {
    "fm_version": (_c_int, []),
    "fm_last_error": (ctypes.c_char_p, []),
    "fm_workspace_size": (_c_int, [_i64, _i64, ctypes.POINTER(_u64)]),
    "fm_fused_newton_schulz": (_c_int, [_vp, _c_int, _i64, _i64, _i64, _vp, _c_int, _vp, _u64, _vp]),
    "fm_workspace_size_batched": (_c_int, [_i64, _i64, _i64, ctypes.POINTER(_u64)]),
    "fm_fused_newton_schulz_batched": (_c_int, [_vp, _c_int, _i64, _i64, _i64, _i64, _i64, _vp,
                                                _i64, _c_int, _vp, _u64, _vp]),
    "fm_newton_schulz_step": (_c_int, [_vp, _i64, _i64, _i64, _vp, _vp, _u64, _vp]),
    "fm_ns_step_debug": (_c_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _u64, _vp]),
    "fm_device_error": (_c_int, [ctypes.POINTER(ctypes.c_uint32)]),
    "fm_selftest_wait_timeout": (_c_int, [_vp]),
    "fm_fused_newton_schulz_noalloc": (_c_int, [_vp, _c_int, _i64, _i64, _i64, _vp, _c_int, _vp]),
    "fm_muon_momentum": (_c_int, [_vp, _vp, _vp, _i64, _c_int, ctypes.c_float, _c_int, _vp]),
    "fm_muon_apply": (_c_int, [_vp, _c_int, _vp, _i64, ctypes.c_float, ctypes.c_float, _vp]),
    "fm_set_gemm_path": (_c_int, [_c_int]),
    "fm_stage_timing": (_c_int, [_c_int]),
    "fm_stage_times": (_c_int, [ctypes.POINTER(ctypes.c_float), ctypes.POINTER(_c_int)]),
    "fm_launch_count": (_c_int, [ctypes.POINTER(ctypes.c_uint64)]),
}

_lib = None
_lock = threading.Lock()


class FusedMuonError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def load() -> ctypes.CDLL:
    """Load (once) and return the native library, raising if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing; build it with `python -m muon_fused.build` "
                    "(there is no fallback implementation)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != FM_OK:
        msg = load().fm_last_error().decode(errors="replace")
        raise FusedMuonError(f"{what} failed (status {rc}): {msg}")


def workspace_bytes(rows: int, cols: int) -> int:
    out = ctypes.c_uint64(0)
    check(load().fm_workspace_size(int(rows), int(cols), ctypes.byref(out)), "fm_workspace_size")
    return int(out.value)


def workspace_bytes_batched(batch: int, rows: int, cols: int) -> int:
    out = ctypes.c_uint64(0)
    check(load().fm_workspace_size_batched(int(batch), int(rows), int(cols), ctypes.byref(out)),
          "fm_workspace_size_batched")
    return int(out.value)


def device_error() -> int:
    code = ctypes.c_uint32(0)
    check(load().fm_device_error(ctypes.byref(code)), "fm_device_error")
    return int(code.value)


STAGES = ("gemm1_syrk", "gemm2_poly", "gemm3_bx", "prep", "fused_ns")


def stage_timing(enable: bool) -> None:
    check(load().fm_stage_timing(1 if enable else 0), "fm_stage_timing")


def stage_times():
    """{stage: (total ms, launches)} since the last read (see fm_stage_times)."""
    ms = (ctypes.c_float * len(STAGES))()
    cnt = (ctypes.c_int * len(STAGES))()
    check(load().fm_stage_times(ms, cnt), "fm_stage_times")
    return {STAGES[i]: (float(ms[i]), int(cnt[i])) for i in range(len(STAGES))}


def launch_count() -> int:
    """Kernels the library has launched in this process (see fm_launch_count)."""
    n = ctypes.c_uint64(0)
    check(load().fm_launch_count(ctypes.byref(n)), "fm_launch_count")
    return int(n.value)


def set_gemm_path(path: int) -> None:
    """0 automatic, 1 single-CTA tiles, 2 CTA-pair tiles, 3/4/5 persistent
    kernel with 128x256 / 128x128 / CTA-pair tiles (see fm_set_gemm_path)."""
    check(load().fm_set_gemm_path(int(path)), "fm_set_gemm_path")
