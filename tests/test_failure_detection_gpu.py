"""Failure detection on the GPU without a fault: a pipeline wait is made to
run out (its loads are withheld) and the kernel must end on its own, report
the timeout through the device error word, and leave the context usable."""

import pytest
import torch

from oracle import ns_oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_recovers(cuda_lib):
    from muon_fused import _lib, fused_newton_schulz

    assert _lib.device_error() == 0
    _lib.check(cuda_lib.fm_selftest_wait_timeout(torch.cuda.current_stream().cuda_stream),
               "fm_selftest_wait_timeout")
    assert _lib.device_error() == 1  # kErrWaitFull: MMA warp gave up waiting for a stage
    assert _lib.device_error() == 0  # reading cleared it
    # the context still works
    G = torch.randn(256, 384, generator=torch.Generator().manual_seed(0)).bfloat16()
    out = fused_newton_schulz(G.cuda(), 5)
    torch.cuda.synchronize()
    assert O.rel_fro(out.cpu(), O.ns_fp32(G, 5)) <= 1e-2
    assert _lib.device_error() == 0


def test_errors_raise_instead_of_falling_back(cuda_lib):
    """The reference swallows every exception and reruns on PyTorch
    (ns_step.py:117-120); here a bad call raises."""
    from muon_fused import _fused_muon_C as _C

    with pytest.raises(RuntimeError, match="bf16"):
        _C.newton_schulz_step(torch.randn(64, 64, device="cuda"))
    with pytest.raises(RuntimeError, match="2D"):
        _C.fused_newton_schulz(torch.randn(2, 3, 4, device="cuda"))
