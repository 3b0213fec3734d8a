"""Build the native library ``muon_fused/libfused_muon.so`` for sm_100a.

The library is plain CUDA C++ behind the C ABI of ``include/fused_muon.h``;
it links only the CUDA runtime (the tensor-map encoder is fetched from the
driver at run time), so it is built with nvcc directly rather than as a torch
extension.  The build is in-tree so the .so travels with the source tree.

Usage: ``python -m muon_fused.build`` (or ``build()`` from Python).
"""

from __future__ import annotations

import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libfused_muon.so")
SOURCES = ["ns_capi.cu"]
DEPS = SOURCES + ["fm_ptx.cuh", "ns_gemm_sm100.cuh", "ns_gemm2_sm100.cuh", "ns_prep.cuh", "ns_fused_sm100.cuh", "ns_fused2_sm100.cuh",
                  "muon_elementwise.cuh"]
HEADER = os.path.join(os.path.dirname(HERE), "include", "fused_muon.h")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the fused_muon library needs the CUDA toolkit to build")
    return cand


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, d) for d in DEPS] + [HEADER]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path."""
    if not force and not _stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", tmp] + [os.path.join(CSRC, s) for s in SOURCES]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
