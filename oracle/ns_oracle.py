"""CPU oracle for the Newton-Schulz / Muon hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker or the timed CPU baseline.
The product path (``muon_fused``) never calls it and has no CPU fallback.

Pinning: ``ns_reference_bf16`` and ``muon_reference_step`` are checked
bit-for-bit against golden outputs of the reference itself
(``tests/golden/make_golden.py`` imports StarrickLiu/fused-muon and records
them; ``tests/test_oracle.py`` replays them).

Contents
--------
ns_reference_bf16   restates muon_fused/ns_step.py:25-55 (identical to
                    benchmarks/reference_muon.py:14-37): bf16 storage, every op
                    rounded to bf16 by torch's CPU kernels.
ns_fp32             the same algorithm in fp32 throughout: the accuracy yardstick
                    (relative Frobenius error <= 1e-2 is the parity gate).
ns_b200_model       the arithmetic of the B200 kernels restated on the CPU: bf16
                    X/A/B storage, fp32 accumulation, fp32 epilogues, B's diagonal
                    kept in fp32 (see muon_fused/csrc/ns_gemm_sm100.cuh).
muon_reference_step restates the Muon branch of muon_fused/optimizer.py:120-163
                    and the AdamW branch :165-200 (= benchmarks/reference_muon.py:94-154).
"""

from __future__ import annotations

import math

import torch

# reference muon_fused/ns_step.py:39
A_COEF, B_COEF, C_COEF = 3.4445, -4.7750, 2.0315


def ns_reference_bf16(G: torch.Tensor, steps: int) -> torch.Tensor:
    """Reference bf16 Newton-Schulz (muon_fused/ns_step.py:25-55), op for op."""
    a, b, c = A_COEF, B_COEF, C_COEF
    X = G.bfloat16()
    if G.size(0) > G.size(1):  # ns_step.py:41-42
        X = X.T
    X = X / (X.norm() + 1e-7)  # ns_step.py:45
    for _ in range(steps):  # ns_step.py:48-51
        A = X @ X.T
        B = b * A + c * A @ A
        X = a * X + B @ X
    if G.size(0) > G.size(1):  # ns_step.py:53-54
        X = X.T
    return X


def ns_fp32(G: torch.Tensor, steps: int) -> torch.Tensor:
    """The reference algorithm computed in fp32 (float64 inputs stay float64)."""
    a, b, c = A_COEF, B_COEF, C_COEF
    dt = torch.float64 if G.dtype == torch.float64 else torch.float32
    X = G.to(dt)
    tall = G.size(0) > G.size(1)
    if tall:
        X = X.T
    X = X / (X.norm() + 1e-7)
    for _ in range(steps):
        A = X @ X.T
        B = b * A + c * (A @ A)
        X = a * X + B @ X
    return X.T if tall else X


def _bf(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def ns_b200_model(G: torch.Tensor, steps: int) -> torch.Tensor:
    """CPU model of the B200 kernels' arithmetic (fp32 math, bf16 storage)."""
    a, b, c = A_COEF, B_COEF, C_COEF
    X = _bf(G.float())
    tall = G.size(0) > G.size(1)
    if tall:
        X = X.T
    X = _bf(X / (X.norm() + 1e-7))
    for _ in range(steps):
        A = _bf(X @ X.T)                       # GEMM1, bf16 store
        P = c * (A @ A) + b * A                # GEMM2 accumulator + epilogue (fp32)
        d = torch.diagonal(P) + a              # fp32 diagonal
        Boff = _bf(P - torch.diag(torch.diagonal(P)))
        X = _bf(d[:, None] * X + Boff @ X)     # GEMM3 + epilogue
    X = X.T if tall else X
    return X.to(torch.bfloat16)


def ns_single_step_reference(X: torch.Tensor) -> torch.Tensor:
    """One bf16 iteration as the reference's tests define it
    (tests/test_correctness.py:37-42)."""
    a, b, c = A_COEF, B_COEF, C_COEF
    A = X @ X.T
    B = b * A + c * A @ A
    return a * X + B @ X


def rel_fro(x: torch.Tensor, ref: torch.Tensor) -> float:
    """Relative Frobenius error ||x - ref|| / ||ref|| in float64."""
    x64, r64 = x.double(), ref.double()
    return float((x64 - r64).norm() / r64.norm())


def max_rel(x: torch.Tensor, ref: torch.Tensor) -> float:
    """The reference tests' metric: max|x - ref| / max|ref|
    (tests/test_correctness.py:96-100)."""
    x32, r32 = x.float(), ref.float()
    return float((x32 - r32).abs().max() / max(r32.abs().max().item(), 1e-6))


def adjust_lr_for_muon(lr: float, shape) -> float:
    """muon_fused/optimizer.py:79-84."""
    A, B = shape[:2]
    return lr * 0.2 * math.sqrt(max(A, B))


@torch.no_grad()
def muon_reference_step(param_groups, state: dict, ns=ns_reference_bf16) -> None:
    """One optimizer step with the reference's semantics (optimizer.py:99-202).

    ``param_groups``: list of dicts with keys params, use_muon, lr, wd,
    momentum, nesterov, ns_steps, adamw_betas, adamw_eps.  ``state`` maps
    id(param) -> per-parameter dict (momentum_buffer / step, moment1, moment2).
    """
    for group in param_groups:
        lr, wd = group["lr"], group["wd"]
        if group.get("use_muon", False):
            mom = group["momentum"]
            for p in group["params"]:
                g = p.grad
                if g is None:
                    continue
                if g.ndim > 2:
                    g = g.view(g.size(0), -1)
                st = state.setdefault(id(p), {})
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(g)
                buf = st["momentum_buffer"]
                buf.mul_(mom).add_(g)
                g = g.add(buf, alpha=mom) if group["nesterov"] else buf
                u = ns(g, group["ns_steps"])
                if u.shape != p.shape:
                    u = u.view_as(p)
                p.data.mul_(1 - lr * wd)
                p.data.add_(u, alpha=-adjust_lr_for_muon(lr, p.shape))
        else:
            beta1, beta2 = group["adamw_betas"]
            eps = group["adamw_eps"]
            for p in group["params"]:
                g = p.grad
                if g is None:
                    continue
                st = state.setdefault(id(p), {})
                if "step" not in st:
                    st["step"] = 0
                    st["moment1"] = torch.zeros_like(g)
                    st["moment2"] = torch.zeros_like(g)
                st["step"] += 1
                step = st["step"]
                buf1, buf2 = st["moment1"], st["moment2"]
                buf1.lerp_(g, 1 - beta1)
                buf2.lerp_(g.square(), 1 - beta2)
                g = buf1 / (eps + buf2.sqrt())
                bc1 = 1 - beta1 ** step
                bc2 = 1 - beta2 ** step
                scale = bc1 / bc2 ** 0.5
                p.data.mul_(1 - lr * wd)
                p.data.add_(g, alpha=-lr / scale)
