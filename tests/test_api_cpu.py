"""Python surface: the reference's names exist, and CPU tensors raise instead
of silently falling back (the reference falls back, ns_step.py:111-123)."""

import pytest
import torch

import muon_fused
from muon_fused import FusedMuon, fused_newton_schulz
from muon_fused import _fused_muon_C as _C


def test_public_names():
    assert muon_fused.__version__ == "0.1.0"
    assert set(["FusedMuon", "fused_newton_schulz"]) <= set(muon_fused.__all__)
    for name in ("newton_schulz_step", "fused_newton_schulz", "workspace_size"):
        assert callable(getattr(_C, name))


def test_cpu_tensor_raises():
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_newton_schulz(torch.randn(8, 8))
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.newton_schulz_step(torch.randn(8, 8).bfloat16())


def test_non_2d_asserts():
    with pytest.raises(AssertionError):
        fused_newton_schulz(torch.randn(2, 3, 4))


def test_workspace_size_bytes():
    assert muon_fused.workspace_size(4096, 4096) == _C.workspace_size(4096, 4096)
    assert muon_fused.workspace_size(4096, 4096) >= 4 * 4096 * 4096 * 2


def test_optimizer_signature_and_adamw_on_cpu():
    """Groups without use_muon run the reference's AdamW branch (no kernels)."""
    p = torch.nn.Parameter(torch.ones(4))
    opt = FusedMuon([p], lr=0.1)
    assert opt.defaults["momentum"] == 0.95 and opt.defaults["nesterov"] is True
    assert opt.defaults["ns_steps"] == 5 and opt.defaults["wd"] == 0.1
    assert opt.defaults["adamw_betas"] == (0.9, 0.95) and opt.defaults["adamw_eps"] == 1e-8
    p.grad = torch.full((4,), 0.5)
    opt.step()
    st = opt.state[p]
    assert st["step"] == 1 and "moment1" in st and "moment2" in st
    assert FusedMuon.adjust_lr_for_muon(0.02, torch.Size([64, 256])) == pytest.approx(0.02 * 0.2 * 16)
