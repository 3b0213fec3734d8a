"""Newton-Schulz orthogonalisation front door.

Same public surface as the reference's ``muon_fused/ns_step.py``:
``fused_newton_schulz(G, steps=5, workspace=None)`` (ns_step.py:85-123) and
``workspace_size(m, n)`` (ns_step.py:61-79).  Differences by design:

* CUDA only.  The reference silently falls back to a PyTorch loop on CPU
  tensors, on a missing extension and on *any* runtime error
  (ns_step.py:111-123); here a CPU tensor or a failing kernel raises.
* ``workspace_size`` returns bytes (the reference's C++ value,
  torch_binding.cu:16-18).  Callers that allocate that many bf16 elements, as
  the reference's optimizer does (optimizer.py:90-92), simply over-allocate.
"""

from __future__ import annotations

import torch

from muon_fused import _fused_muon_C as _C

# Newton-Schulz quintic coefficients (reference ns_step.py:39).
NS_COEFFS = (3.4445, -4.7750, 2.0315)


def workspace_size(m: int, n: int) -> int:
    """Bytes of device workspace needed for an (m, n) gradient matrix."""
    return _C.workspace_size(m, n)


def fused_newton_schulz(
    G: torch.Tensor,
    steps: int = 5,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """Approximate orthogonal factor of ``G`` by ``steps`` quintic
    Newton-Schulz iterations; returns bf16 with ``G``'s shape.

    Args:
        G: 2-D CUDA tensor of any floating dtype (cast to bf16 internally).
        steps: number of iterations (default 5).
        workspace: optional pre-allocated CUDA buffer of at least
            ``workspace_size(*G.shape)`` bytes; reused across calls.
    """
    assert G.ndim == 2, f"Expected 2-D tensor, got {G.ndim}-D"
    if not G.is_cuda:
        raise RuntimeError(
            "fused_newton_schulz needs a CUDA tensor; this build has no CPU fallback")
    return _C.fused_newton_schulz(G, steps, workspace)
