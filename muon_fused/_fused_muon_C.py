"""Tensor-level wrappers over the C ABI, mirroring the reference's pybind
module ``muon_fused._fused_muon_C`` (csrc/torch_binding.cu:125-135): the same
names, argument meanings and error behaviour (``RuntimeError`` on bad input),
plus ``ns_step_debug`` for symmetry tests.

All calls run on torch's current CUDA stream and never synchronise the host.
"""

from __future__ import annotations

import torch

from muon_fused import _lib

_DTYPE_CODE = {
    torch.bfloat16: _lib.FM_DT_BF16,
    torch.float16: _lib.FM_DT_F16,
    torch.float32: _lib.FM_DT_F32,
    torch.float64: _lib.FM_DT_F64,
}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (fused_muon has no CPU implementation)")


def workspace_size(m: int, n: int) -> int:
    """Workspace size in bytes for an (m, n) matrix (either orientation).

    Reference: csrc/torch_binding.cu:16-18 (``_C.workspace_size``)."""
    return _lib.workspace_bytes(m, n)


def _workspace(G: torch.Tensor, rows: int, cols: int, workspace):
    need = _lib.workspace_bytes(rows, cols)
    if workspace is None:
        return torch.empty(need, dtype=torch.uint8, device=G.device), need
    _check_cuda(workspace, "workspace")
    if workspace.device != G.device:
        raise RuntimeError("workspace must be on the same device as the input")
    if workspace.nbytes < need:
        # Same policy as the reference (torch_binding.cu:95-102): a too-small
        # workspace is replaced by a fresh allocation.
        return torch.empty(need, dtype=torch.uint8, device=G.device), need
    return workspace, workspace.nbytes


def fused_newton_schulz(G: torch.Tensor, steps: int = 5, workspace=None) -> torch.Tensor:
    """Full Newton-Schulz iteration; bf16 result with G's shape.

    Reference: csrc/torch_binding.cu:58-123."""
    _check_cuda(G, "G")
    if G.dim() != 2:
        raise RuntimeError("G must be 2D")
    if G.dtype not in _DTYPE_CODE:
        raise RuntimeError(f"unsupported dtype {G.dtype}; expected a floating type")
    if G.stride(1) != 1:
        G = G.contiguous()
    rows, cols = G.shape
    out = torch.empty((rows, cols), dtype=torch.bfloat16, device=G.device)
    if G.numel() == 0:
        return out
    ws, ws_bytes = _workspace(G, rows, cols, workspace)
    with torch.cuda.device(G.device):
        _lib.check(
            _lib.load().fm_fused_newton_schulz(
                G.data_ptr(), _DTYPE_CODE[G.dtype], rows, cols, G.stride(0), out.data_ptr(),
                int(steps), ws.data_ptr(), ws_bytes, _stream(G)),
            "fm_fused_newton_schulz")
    return out


def workspace_size_batched(batch: int, m: int, n: int) -> int:
    """Workspace bytes for ``batch`` same-shape (m, n) matrices."""
    return _lib.workspace_bytes_batched(batch, m, n)


def fused_newton_schulz_batched(G: torch.Tensor, steps: int = 5, workspace=None,
                                out: torch.Tensor | None = None) -> torch.Tensor:
    """Newton-Schulz on each matrix of a (batch, rows, cols) tensor in one set of
    GEMM launches; returns a bf16 (batch, rows, cols) tensor (or writes ``out``,
    which must be a contiguous bf16 tensor of that shape)."""
    _check_cuda(G, "G")
    if G.dim() != 3:
        raise RuntimeError("G must be 3D (batch, rows, cols)")
    if G.dtype not in _DTYPE_CODE:
        raise RuntimeError(f"unsupported dtype {G.dtype}; expected a floating type")
    if G.stride(2) != 1 or G.stride(0) < G.shape[1] * G.stride(1):
        G = G.contiguous()
    batch, rows, cols = G.shape
    if out is None:
        out = torch.empty((batch, rows, cols), dtype=torch.bfloat16, device=G.device)
    elif (out.shape != G.shape or out.dtype != torch.bfloat16 or not out.is_contiguous()
          or out.device != G.device):
        raise RuntimeError("out must be a contiguous bf16 tensor shaped like G on its device")
    if G.numel() == 0:
        return out
    need = _lib.workspace_bytes_batched(batch, rows, cols)
    if workspace is None or workspace.nbytes < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=G.device)
    with torch.cuda.device(G.device):
        _lib.check(
            _lib.load().fm_fused_newton_schulz_batched(
                G.data_ptr(), _DTYPE_CODE[G.dtype], batch, rows, cols, G.stride(1), G.stride(0),
                out.data_ptr(), rows * cols, int(steps), workspace.data_ptr(), workspace.nbytes,
                _stream(G)),
            "fm_fused_newton_schulz_batched")
    return out


def newton_schulz_step(X: torch.Tensor, workspace=None) -> torch.Tensor:
    """One iteration on a normalised bf16 matrix: (aI + bA + cA²)·X, A = X·Xᵀ.

    Reference: csrc/torch_binding.cu:22-54 (``_C.newton_schulz_step``)."""
    _check_cuda(X, "X")
    if X.dim() != 2:
        raise RuntimeError(f"X must be 2D, got {X.dim()}D")
    if X.dtype != torch.bfloat16:
        raise RuntimeError("X must be bf16")
    if not X.is_contiguous():
        raise RuntimeError("X must be contiguous")
    m, n = X.shape
    X_new = torch.empty_like(X)
    ws, ws_bytes = _workspace(X, m, max(m, n), workspace)
    with torch.cuda.device(X.device):
        _lib.check(
            _lib.load().fm_newton_schulz_step(
                X.data_ptr(), m, n, X.stride(0), X_new.data_ptr(), ws.data_ptr(), ws_bytes,
                _stream(X)),
            "fm_newton_schulz_step")
    return X_new


def ns_step_debug(X: torch.Tensor, workspace=None):
    """One iteration returning ``(A, Boff, diag, X_new)``: A = X·Xᵀ (bf16),
    Boff = off-diagonal of b·A + c·A² (bf16, zero diagonal), diag = a +
    diagonal of b·A + c·A² (fp32), X_new = diag ⊙ X + Boff·X (bf16)."""
    _check_cuda(X, "X")
    if X.dim() != 2 or X.dtype != torch.bfloat16 or not X.is_contiguous():
        raise RuntimeError("X must be a contiguous 2D bf16 tensor")
    m, n = X.shape
    A = torch.empty((m, m), dtype=torch.bfloat16, device=X.device)
    B = torch.empty_like(A)
    d = torch.empty(m, dtype=torch.float32, device=X.device)
    X_new = torch.empty_like(X)
    ws, ws_bytes = _workspace(X, m, max(m, n), workspace)
    with torch.cuda.device(X.device):
        _lib.check(
            _lib.load().fm_ns_step_debug(
                X.data_ptr(), m, n, X.stride(0), A.data_ptr(), B.data_ptr(), d.data_ptr(),
                X_new.data_ptr(), ws.data_ptr(), ws_bytes, _stream(X)),
            "fm_ns_step_debug")
    return A, B, d, X_new
