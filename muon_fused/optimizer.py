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
* Momentum state is kept only by the owning rank, so ``state_dict`` is
  rank-local when sharded until ``consolidate_state_dict()`` broadcasts every
  buffer from its owner; keys are the reference's ``momentum_buffer``.
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch.optim import Optimizer

from muon_fused import _fused_muon_C as _C
from muon_fused import _lib
from muon_fused.ns_step import workspace_size

# Parameter / gradient dtypes the fused elementwise kernels handle.
_EW_DTYPES = {torch.float32: _lib.FM_DT_F32, torch.bfloat16: _lib.FM_DT_BF16,
              torch.float16: _lib.FM_DT_F16}


def _ns_batched(G: torch.Tensor, steps: int, workspace: torch.Tensor, out: torch.Tensor):
    """Batched Newton-Schulz used by the optimizer (module level so a test can
    substitute a CPU implementation in a gloo child process)."""
    return _C.fused_newton_schulz_batched(G, steps, workspace, out=out)


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
        batch_bytes: device memory one batched Newton-Schulz call may use for
            its inputs, outputs and workspace (default 4 GiB); same-shape
            matrices are batched up to this budget.
        collective: how a sharded step shares the updates: ``"nccl"`` (bucketed
            all-gather of the bf16 updates, then every rank applies every
            update) or ``"param_gather"`` (each owner applies its own updates,
            then the bucket's parameters are all-gathered in place; the
            parameters' ``.data`` are moved into per-bucket flat buffers for
            this, see ``sharding.ParamStore``).  Both give bit-identical
            parameters.
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
        batch_bytes: int = 4 << 30,
        collective: str = "nccl",
    ):
        defaults: dict[str, Any] = dict(
            lr=lr, wd=wd, momentum=momentum, nesterov=nesterov, ns_steps=ns_steps,
            adamw_betas=adamw_betas, adamw_eps=adamw_eps,
        )
        super().__init__(param_groups, defaults)
        self._workspaces: dict[tuple, torch.Tensor] = {}
        self._process_group = process_group
        self._bucket_bytes = int(bucket_bytes)
        self._batch_bytes = int(batch_bytes)
        self._plans: dict[tuple, Any] = {}
        self._arena: dict[torch.device, torch.Tensor] = {}
        if collective not in ("nccl", "param_gather"):
            raise ValueError(f"collective must be 'nccl' or 'param_gather', got {collective!r}")
        self._collective = collective
        self._stores: dict[tuple, Any] = {}
        # id(group) -> (params, owner rank per param, momentum dtype per param)
        # of the group's last sharded step (consolidate_state_dict)
        self._owners: dict[int, tuple] = {}

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
    def _momentum_into(self, p: torch.Tensor, g: torch.Tensor, dst: torch.Tensor, momentum: float,
                       nesterov: bool) -> None:
        """buf ← μ·buf + g; dst ← bf16(g + μ·buf) (nesterov) or bf16(buf)
        (optimizer.py:139-149).

        On CUDA this is one fused kernel (fm_muon_momentum) writing the bf16
        Newton-Schulz input straight into ``dst``; the buffer is bit-identical
        to the reference's torch ops.  CPU tensors (no Newton-Schulz path
        exists for them) keep the reference's torch ops."""
        state = self.state[p]
        if "momentum_buffer" not in state:
            state["momentum_buffer"] = torch.zeros_like(g)
        buf = state["momentum_buffer"]
        dt = _EW_DTYPES.get(g.dtype)
        if g.is_cuda and dt is not None and buf.is_contiguous() and dst.is_contiguous():
            gc = g if g.is_contiguous() else g.contiguous()
            with torch.cuda.device(g.device):
                _lib.check(_lib.load().fm_muon_momentum(
                    buf.data_ptr(), gc.data_ptr(), dst.data_ptr(), g.numel(), dt,
                    float(momentum), 1 if nesterov else 0,
                    torch.cuda.current_stream(g.device).cuda_stream), "fm_muon_momentum")
            return
        buf.mul_(momentum).add_(g)
        dst.copy_(g.add(buf, alpha=momentum) if nesterov else buf)

    def _scratch(self, device: torch.device, nbytes: int) -> torch.Tensor:
        """One reusable device buffer per device for batch inputs, outputs and
        the Newton-Schulz workspace.  Reuse is safe because every user is
        ordered on the same stream."""
        buf = self._arena.get(device)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
            self._arena[device] = buf
        return buf

    def _batch_limit(self, rows: int, cols: int) -> int:
        """Matrices per batched call so inputs, outputs and workspace of one
        batch stay within ``batch_bytes``."""
        per = _C.workspace_size_batched(1, rows, cols) + 4 * rows * cols
        return max(1, min(64, self._batch_bytes // per))

    def _orthogonalise_batch(self, params, group, out=None) -> torch.Tensor:
        """Momentum + Newton-Schulz for same-shape parameters in one batched
        call; returns (B, rows, cols) bf16 updates (written into ``out`` when
        given, e.g. a slice of the all-gather send buffer)."""
        g0 = params[0].grad
        rows = g0.size(0)
        cols = g0.numel() // rows
        B = len(params)
        dev = g0.device
        n_el = B * rows * cols
        dir_bytes = (2 * n_el + 255) // 256 * 256
        ws_bytes = _C.workspace_size_batched(B, rows, cols)
        out_bytes = 0 if out is not None else (2 * n_el + 255) // 256 * 256
        arena = self._scratch(dev, dir_bytes + out_bytes + ws_bytes)
        dirs = arena[:2 * n_el].view(torch.bfloat16).view(B, rows, cols)
        if out is None:
            out = arena[dir_bytes:dir_bytes + 2 * n_el].view(torch.bfloat16).view(B, rows, cols)
        ws = arena[dir_bytes + out_bytes:dir_bytes + out_bytes + ws_bytes]
        for b, p in enumerate(params):
            g = p.grad
            if g.ndim > 2:
                g = g.view(g.size(0), -1)
            self._momentum_into(p, g, dirs[b], group["momentum"], group["nesterov"])
        _ns_batched(dirs, group["ns_steps"], ws, out)
        return out

    @staticmethod
    def _apply_update(p: torch.Tensor, u: torch.Tensor, lr: float, wd: float) -> None:
        """p ← p·(1 − lr·wd) − lr'·u (optimizer.py:157-163), one fused pass
        (fm_muon_apply) on CUDA, bit-identical to the two torch ops."""
        if u.shape != p.shape:
            u = u.view_as(p)
        alpha = -FusedMuon.adjust_lr_for_muon(lr, p.shape)
        dt = _EW_DTYPES.get(p.dtype)
        data = p.data
        if (data.is_cuda and dt is not None and data.is_contiguous() and u.is_contiguous()
                and u.dtype == torch.bfloat16):
            with torch.cuda.device(data.device):
                _lib.check(_lib.load().fm_muon_apply(
                    data.data_ptr(), dt, u.data_ptr(), data.numel(), float(1 - lr * wd),
                    float(alpha), torch.cuda.current_stream(data.device).cuda_stream),
                    "fm_muon_apply")
            return
        data.mul_(1 - lr * wd)
        data.add_(u, alpha=alpha)

    def _muon_group_local(self, group) -> None:
        """All matrices on this process: same-shape parameters are batched
        into one Newton-Schulz call (the reference loops one matrix at a time,
        optimizer.py:128-163)."""
        by_shape: dict[tuple, list] = {}
        for p in group["params"]:
            if p.grad is None:
                continue
            key = (p.grad.device, p.shape[0], p.grad.numel() // p.shape[0])
            by_shape.setdefault(key, []).append(p)
        for (_, rows, cols), plist in by_shape.items():
            lim = self._batch_limit(rows, cols)
            for k in range(0, len(plist), lim):
                chunk = plist[k:k + lim]
                out = self._orthogonalise_batch(chunk, group)
                for b, p in enumerate(chunk):
                    self._apply_update(p, out[b], group["lr"], group["wd"])

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

        self._owners[id(group)] = (params, list(plan.owner), [p.grad.dtype for p in params])
        for p, r in zip(params, plan.owner):
            if r != rank and p in self.state:  # e.g. after loading a consolidated checkpoint
                self.state[p].pop("momentum_buffer", None)

        def compute(indices, out) -> None:
            rows, cols = out.shape[1], out.shape[2]
            lim = self._batch_limit(rows, cols)
            for k in range(0, len(indices), lim):
                self._orthogonalise_batch([params[i] for i in indices[k:k + lim]], group,
                                          out[k:k + lim])

        def apply(i: int, u: torch.Tensor) -> None:
            self._apply_update(params[i], u, group["lr"], group["wd"])

        dev = params[0].device
        store = self._stores.get(key)
        if self._collective == "param_gather" and (store is not None
                                                   or sharding.ParamStore.supports(params)):
            # supports() is checked before the store exists: afterwards the
            # parameters deliberately share the store's flat buffers
            if store is None:
                store = sharding.ParamStore(plan, params, dev)
                self._stores[key] = store
            store.bind(params)
            sharding.run_sharded_param_gather(store, rank, pg, compute, apply)
            return
        sharding.run_sharded(plan, rank, pg, dev, compute, apply)

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
    def consolidate_state_dict(self) -> None:
        """Make every rank's optimizer state complete after sharded steps.

        Under sharding a matrix's momentum buffer lives only on the rank that
        owns it.  This broadcasts every buffer from its owner, so that
        ``state_dict()`` on any rank then holds the same keys and values as a
        single-process run (and as the reference optimizer,
        optimizer.py:140-141): ready to save, and to load into a run with any
        number of ranks (a sharded step keeps only the buffers its rank owns).
        A collective: every rank of the process group calls it.  Without
        sharding it does nothing.
        """
        pg, rank, world = self._world()
        if world <= 1:
            return
        import torch.distributed as dist

        for group in self.param_groups:
            rec = self._owners.get(id(group))
            if rec is None:
                continue
            params, owner, dtypes = rec
            for p, r, dt in zip(params, owner, dtypes):
                st = self.state[p]
                buf = st.get("momentum_buffer") if r == rank else None
                if buf is None:
                    # the buffer has the gradient's 2-D view shape (see _orthogonalise_batch)
                    shape = (p.shape[0], p.numel() // p.shape[0]) if p.ndim > 2 else p.shape
                    buf = torch.empty(shape, dtype=dt, device=p.device)
                    st["momentum_buffer"] = buf
                src = dist.get_global_rank(pg, r) if pg is not None else r
                dist.broadcast(buf, src=src, group=pg)

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
