"""FusedMuon — Muon with the B200 Newton-Schulz engine.

Same constructor, defaults, state keys and group semantics as the reference
(muon_fused/optimizer.py:51-202):

* groups with ``use_muon=True`` run SGD-momentum (nesterov by default), the
  Newton-Schulz orthogonalisation, decoupled weight decay and the
  ``0.2·sqrt(max(A, B))`` learning-rate scale (optimizer.py:120-163);
* every other group runs the reference's AdamW variant unchanged
  (optimizer.py:165-200) — including the quirk that a plain parameter list
  has no ``use_muon`` key and therefore takes the AdamW branch.

B200-specific behaviour:

* Parameters of a Muon group are processed through ``muon_fused.sharding``:
  under ``torch.distributed`` with world size > 1 each rank orthogonalises
  only the matrices it owns (FLOP-balanced assignment) and the bf16 updates
  are all-gathered over NCCL; with one process everything is local.
* Momentum state is kept only by the owning rank (``state_dict`` is therefore
  rank-local when sharded; keys are the reference's ``momentum_buffer``).
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch.optim import Optimizer

from muon_fused.ns_step import fused_newton_schulz, workspace_size


class FusedMuon(Optimizer):
    """Muon optimizer with fused Newton-Schulz orthogonalisation.

    Args:
        param_groups: iterable of parameters or of group dicts; groups with
            ``"use_muon": True`` take the Muon path, all others AdamW.
        lr: base learning rate (default ``1e-3``).
        wd: decoupled weight decay (default ``0.1``).
        momentum: SGD momentum of Muon groups (default ``0.95``).
        nesterov: Nesterov momentum (default ``True``).
        ns_steps: Newton-Schulz iterations (default ``5``).
        adamw_betas: AdamW betas (default ``(0.9, 0.95)``).
        adamw_eps: AdamW epsilon (default ``1e-8``).
        process_group: process group to shard Muon work over; defaults to
            the world group when ``torch.distributed`` is initialised.
        bucket_bytes: size of each all-gather bucket of packed updates when
            sharded (default 256 MiB).
    """

    def __init__(
        self,
        param_groups,
        lr: float = 1e-3,
        wd: float = 0.1,
        momentum: float = 0.95,
        nesterov: bool = True,
        ns_steps: int = 5,
        adamw_betas: tuple[float, float] = (0.9, 0.95),
        adamw_eps: float = 1e-8,
        process_group=None,
        bucket_bytes: int = 256 << 20,
    ):
        defaults: dict[str, Any] = dict(
            lr=lr, wd=wd, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
            adamw_betas=adamw_betas, adamw_eps=adamw_eps,
        )
        super().__init__(param_groups, defaults)
        self._workspaces: dict[tuple, torch.Tensor] = {}
        self._process_group = process_group
        self._bucket_bytes = int(bucket_bytes)
        self._plans: dict[tuple, Any] = {}

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def adjust_lr_for_muon(lr: float, param_shape: torch.Size) -> float:
        """``lr · 0.2 · sqrt(max(A, B))`` over the first two dims (optimizer.py:79-84)."""
        A, B = param_shape[:2]
        return lr * 0.2 * math.sqrt(max(A, B))

    def _get_workspace(self, m: int, n: int, device: torch.device) -> torch.Tensor:
        """Cached workspace per (device, orientation-free shape) (optimizer.py:86-94)."""
        key = (device, min(m, n), max(m, n))
        ws = self._workspaces.get(key)
        if ws is None:
            ws = torch.empty(workspace_size(m, n), dtype=torch.uint8, device=device)
            self._workspaces[key] = ws
        return ws

    def _world(self):
        import torch.distributed as dist

        if not (dist.is_available() and dist.is_initialized()):
            return None, 0, 1
        pg = self._process_group
        return pg, dist.get_rank(pg), dist.get_world_size(pg)

    # ------------------------------------------------------------------ Muon
    def _momentum_direction(self, p: torch.Tensor, g: torch.Tensor, momentum: float,
                            nesterov: bool) -> torch.Tensor:
        """buf ← μ·buf + g; returns g + μ·buf (nesterov) or buf (optimizer.py:139-149)."""
        state = self.state[p]
        if "momentum_buffer" not in state:
            state["momentum_buffer"] = torch.zeros_like(g)
        buf = state["momentum_buffer"]
        buf.mul_(momentum).add_(g)
        return g.add(buf, alpha=momentum) if nesterov else buf

    def _orthogonalise(self, p: torch.Tensor, group) -> torch.Tensor:
        g = p.grad
        if g.ndim > 2:
            g = g.view(g.size(0), -1)
        d = self._momentum_direction(p, g, group["momentum"], group["nesterov"])
        ws = self._get_workspace(d.size(0), d.size(1), d.device)
        return fused_newton_schulz(d, steps=group["ns_steps"], workspace=ws)

    @staticmethod
    def _apply_update(p: torch.Tensor, u: torch.Tensor, lr: float, wd: float) -> None:
        """p ← p·(1 − lr·wd) − lr'·u (optimizer.py:157-163)."""
        if u.shape != p.shape:
            u = u.view_as(p)
        p.data.mul_(1 - lr * wd)
        p.data.add_(u, alpha=-FusedMuon.adjust_lr_for_muon(lr, p.shape))

    def _muon_group_local(self, group) -> None:
        for p in group["params"]:
            if p.grad is None:
                continue
            u = self._orthogonalise(p, group)
            self._apply_update(p, u, group["lr"], group["wd"])

    def _muon_group_sharded(self, group, pg, rank: int, world: int) -> None:
        from muon_fused import sharding

        params = [p for p in group["params"] if p.grad is not None]
        if not params:
            return
        key = (id(group), tuple(id(p) for p in params), world)
        plan = self._plans.get(key)
        if plan is None:
            plan = sharding.ShardPlan.build([tuple(p.shape) for p in params], world,
                                            self._bucket_bytes)
            self._plans[key] = plan

        def compute(i: int) -> torch.Tensor:
            return self._orthogonalise(params[i], group)

        def apply(i: int, u: torch.Tensor) -> None:
            self._apply_update(params[i], u, group["lr"], group["wd"])

        sharding.run_sharded(plan, rank, pg, params[0].device, compute, apply)

    # ------------------------------------------------------------------ AdamW
    def _adamw_group(self, group) -> None:
        """Reference AdamW branch, unchanged (optimizer.py:165-200)."""
        lr, wd = group["lr"], group["wd"]
        beta1, beta2 = group["adamw_betas"]
        eps: float = group["adamw_eps"]
        for p in group["params"]:
            g = p.grad
            if g is None:
                continue
            state = self.state[p]
            if "step" not in state:
                state["step"] = 0
                state["moment1"] = torch.zeros_like(g)
                state["moment2"] = torch.zeros_like(g)
            state["step"] += 1
            step: int = state["step"]
            buf1, buf2 = state["moment1"], state["moment2"]
            buf1.lerp_(g, 1 - beta1)
            buf2.lerp_(g.square(), 1 - beta2)
            g = buf1 / (eps + buf2.sqrt())
            bias_correction1 = 1 - beta1 ** step
            bias_correction2 = 1 - beta2 ** step
            scale = bias_correction1 / bias_correction2 ** 0.5
            p.data.mul_(1 - lr * wd)
            p.data.add_(g, alpha=-lr / scale)

    # ------------------------------------------------------------------ step
    @torch.no_grad()
    def step(self, closure=None):
        """One optimisation step (optimizer.py:99-202)."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        pg, rank, world = self._world()
        for group in self.param_groups:
            if group.get("use_muon", False):
                if world > 1:
                    self._muon_group_sharded(group, pg, rank, world)
                else:
                    self._muon_group_local(group)
            else:
                self._adamw_group(group)
        return loss
