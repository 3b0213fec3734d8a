"""The persistent Newton-Schulz kernel (all iterations in one launch, phases
ordered by completion counters instead of kernel boundaries).

Its tiles are the single-CTA kernels' tiles and its epilogues are the same
code, so every output element is the same fp32 accumulation in the same
K order: the gate against the one-launch-per-GEMM single-CTA path (which
never splits K) is bit equality, for 128x256 and 128x128 tiles, wide, tall,
ragged and batched inputs and several step counts.  The fp32 gate (relative
Frobenius <= 1e-2) is checked as well, and no bounded wait may have run out.
"""

import pytest
import torch

from oracle import ns_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _with_path(path, fn):
    from muon_fused import _lib

    _lib.set_gemm_path(path)
    try:
        out = fn()
        torch.cuda.synchronize()
        return out
    finally:
        _lib.set_gemm_path(0)


@pytest.mark.parametrize("path", [3, 4])
@pytest.mark.parametrize("shape", [(896, 1152), (1152, 896), (256, 384), (129, 257), (1, 64),
                                   (2048, 2048), (1024, 4096), (2560, 2560), (4096, 4096)])
def test_fused_bit_identical_to_single_cta(cuda_lib, path, shape):
    from muon_fused import _lib, fused_newton_schulz

    G = torch.randn(*shape, generator=torch.Generator().manual_seed(sum(shape))).bfloat16()
    Gd = G.to(DEV)
    want = _with_path(1, lambda: fused_newton_schulz(Gd, 5))
    got = _with_path(path, lambda: fused_newton_schulz(Gd, 5))
    assert torch.equal(got, want), shape
    if shape[0] * shape[1] <= 1 << 21:
        assert O.rel_fro(got.cpu(), O.ns_fp32(G, 5)) <= 1e-2
    assert _lib.device_error() == 0


@pytest.mark.parametrize("path", [3, 4])
@pytest.mark.parametrize("steps", [1, 2, 7])
def test_fused_step_counts(cuda_lib, path, steps):
    from muon_fused import fused_newton_schulz

    G = torch.randn(640, 1536, generator=torch.Generator().manual_seed(steps)).bfloat16().to(DEV)
    want = _with_path(1, lambda: fused_newton_schulz(G, steps))
    got = _with_path(path, lambda: fused_newton_schulz(G, steps))
    assert torch.equal(got, want)


@pytest.mark.parametrize("path", [3, 4])
@pytest.mark.parametrize("b,rows,cols", [(4, 512, 2048), (3, 1152, 896), (8, 256, 512)])
def test_fused_batched(cuda_lib, path, b, rows, cols):
    """A batch in one persistent launch equals each matrix run alone on the
    single-CTA path."""
    from muon_fused import _fused_muon_C as _C
    from muon_fused import _lib

    G = torch.randn(b, rows, cols, generator=torch.Generator().manual_seed(rows)).bfloat16()
    Gd = G.to(DEV)
    got = _with_path(path, lambda: _C.fused_newton_schulz_batched(Gd, 5))
    for i in range(b):
        want = _with_path(1, lambda: _C.fused_newton_schulz(Gd[i], 5))
        assert torch.equal(got[i], want), i
    assert _lib.device_error() == 0


def test_fused_repeated_calls_reuse_workspace(cuda_lib):
    """Back-to-back calls on one workspace (the phase counters are re-zeroed
    per call) stay deterministic."""
    from muon_fused import fused_newton_schulz, workspace_size

    G = torch.randn(1536, 2048, generator=torch.Generator().manual_seed(5)).bfloat16().to(DEV)
    ws = torch.empty(workspace_size(1536, 2048), dtype=torch.uint8, device=DEV)
    outs = _with_path(3, lambda: [fused_newton_schulz(G, 5, ws) for _ in range(4)])
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


@pytest.mark.parametrize("shape", [(2560, 2560), (3072, 4096), (4096, 4096), (1536, 2048),
                                   (2304, 3000), (4096, 2560), (300, 700)])
def test_fused_pair_bit_identical(cuda_lib, shape):
    """The CTA-pair persistent kernel (path 5: 256x256 tiles, the next
    iteration's X·Xᵀ tiles start on finished row blocks of X') equals the
    single-CTA per-GEMM path bit for bit: same per-element accumulation, and
    neither splits K.  Square, wide, tall (transposed output), ragged."""
    from muon_fused import _lib, fused_newton_schulz

    G = torch.randn(*shape, generator=torch.Generator().manual_seed(sum(shape) + 1)).bfloat16()
    Gd = G.to(DEV)
    want = _with_path(1, lambda: fused_newton_schulz(Gd, 5))
    got = _with_path(5, lambda: fused_newton_schulz(Gd, 5))
    assert torch.equal(got, want), shape
    assert _lib.device_error() == 0


@pytest.mark.parametrize("steps", [1, 2, 7])
def test_fused_pair_step_counts_and_batch(cuda_lib, steps):
    from muon_fused import _fused_muon_C as _C

    G = torch.randn(3, 1280, 2304, generator=torch.Generator().manual_seed(steps)).bfloat16()
    Gd = G.to(DEV)
    got = _with_path(5, lambda: _C.fused_newton_schulz_batched(Gd, steps))
    for i in range(3):
        want = _with_path(1, lambda: _C.fused_newton_schulz(Gd[i], steps))
        assert torch.equal(got[i], want), i
