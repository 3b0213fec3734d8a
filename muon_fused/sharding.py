"""Matrix-sharded Muon step across the ranks of a process group.

The reference runs every parameter's momentum + Newton-Schulz on every
process (muon_fused/optimizer.py:128-163, no collectives at all).  Each
matrix's update is independent, so here:

1. ``ShardPlan.build`` assigns every Muon matrix to one owner rank with a
   deterministic FLOP-balanced longest-processing-time rule (all ranks compute
   the same table from the shapes alone, no communication);
2. each rank runs momentum + Newton-Schulz only for the matrices it owns and
   packs the bf16 updates into per-bucket send buffers;
3. each bucket is all-gathered (``all_gather_into_tensor`` over NCCL; a list
   ``all_gather`` on gloo) as soon as it is packed, so the transfer of bucket
   k overlaps the Newton-Schulz work of bucket k+1;
4. every rank then applies the decay + update to every parameter from the
   gathered buffers (``collective="nccl"``), or — ``collective="param_gather"``
   — each owner applies its own updates in place and the bucket's parameters
   themselves are all-gathered in place into every rank's parameter storage
   (``ParamStore``), so non-owners do no apply pass at all.

Gradients must already be identical on all ranks (data parallel after the
gradient all-reduce), which is what makes the owner's update the update.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


def ns_flops(shape, steps: int = 5) -> float:
    """Dense-equivalent FLOPs of ``steps`` Newton-Schulz iterations on a matrix
    (the reference's count 4m²n + 2m³ per iteration, m = min dim)."""
    rows = int(shape[0])
    cols = 1
    for s in shape[1:]:
        cols *= int(s)
    m, n = min(rows, cols), max(rows, cols)
    return steps * (4.0 * m * m * n + 2.0 * m ** 3)


def numel(shape) -> int:
    out = 1
    for s in shape:
        out *= int(s)
    return out


@dataclass
class ShardPlan:
    """Owner table and bucketed packing of one group's matrices."""

    world: int
    owner: list[int]  # matrix index -> rank
    # buckets[k][r] = list of (matrix index, offset) packed by rank r in bucket k
    buckets: list[list[list[tuple[int, int]]]] = field(default_factory=list)
    bucket_numel: list[int] = field(default_factory=list)  # padded per-rank size of bucket k
    shapes: list[tuple] = field(default_factory=list)

    @staticmethod
    def assign(shapes, world: int) -> list[int]:
        """LPT: heaviest matrix first onto the least-loaded rank (ties: lower
        index first, lower rank first)."""
        order = sorted(range(len(shapes)), key=lambda i: (-ns_flops(shapes[i]), i))
        load = [0.0] * world
        owner = [0] * len(shapes)
        for i in order:
            r = min(range(world), key=lambda k: (load[k], k))
            owner[i] = r
            load[r] += ns_flops(shapes[i])
        return owner

    @classmethod
    def build(cls, shapes, world: int, bucket_bytes: int = 256 << 20) -> "ShardPlan":
        shapes = [tuple(int(x) for x in s) for s in shapes]
        owner = cls.assign(shapes, world)
        cap = max(1, bucket_bytes // 2)  # bf16 elements per rank per bucket
        per_rank_chunks: list[list[list[tuple[int, int]]]] = []
        for r in range(world):
            mine = [i for i in range(len(shapes)) if owner[i] == r]
            # heaviest first, so the first buckets carry the long Newton-Schulz
            # calls; equal shapes adjacent so they pack into one batched call
            mine.sort(key=lambda i: (-ns_flops(shapes[i]), shapes[i], i))
            chunks, cur, used = [], [], 0
            for i in mine:
                sz = numel(shapes[i])
                if cur and used + sz > cap:
                    chunks.append(cur)
                    cur, used = [], 0
                cur.append((i, used))
                used += sz
            if cur:
                chunks.append(cur)
            per_rank_chunks.append(chunks)
        nb = max((len(c) for c in per_rank_chunks), default=0)
        buckets, sizes = [], []
        for k in range(nb):
            row = [per_rank_chunks[r][k] if k < len(per_rank_chunks[r]) else [] for r in range(world)]
            size = max((off + numel(shapes[i]) for r in range(world) for i, off in row[r][-1:]),
                       default=0)
            buckets.append(row)
            sizes.append(size)
        return cls(world=world, owner=owner, buckets=buckets, bucket_numel=sizes, shapes=shapes)

    def owned(self, rank: int) -> list[int]:
        return [i for i, r in enumerate(self.owner) if r == rank]


def _all_gather(out: torch.Tensor, inp: torch.Tensor, pg, world: int):
    import torch.distributed as dist

    if dist.get_backend(pg) == "nccl":
        return dist.all_gather_into_tensor(out, inp, group=pg, async_op=True)
    return dist.all_gather(list(out.chunk(world)), inp, group=pg, async_op=True)


def run_sharded(plan: ShardPlan, rank: int, pg, device, compute, apply) -> None:
    """Execute one sharded step.

    ``compute(indices, out)`` writes the bf16 updates of the same-shape
    matrices ``indices`` (owned by this rank, packed back to back in the send
    buffer) into ``out``, a (len(indices), rows, cols) view of that buffer;
    ``apply(i, u)`` applies an update to parameter i (called on every rank,
    in matrix order within each bucket).
    """
    world = plan.world
    pending = []
    for k, row in enumerate(plan.buckets):
        size = plan.bucket_numel[k]
        if size == 0:
            continue
        send = torch.empty(size, dtype=torch.bfloat16, device=device)
        mine = row[rank]
        for idx, off0, n, shape in _runs(plan, mine):
            rows = shape[0]
            cols = numel(shape) // rows
            compute(idx, send[off0:off0 + n * rows * cols].view(n, rows, cols))
        used = max((off + numel(plan.shapes[i]) for i, off in mine[-1:]), default=0)
        if used < size:
            send[used:].zero_()  # padding up to the largest rank's share
        recv = torch.empty(world * size, dtype=torch.bfloat16, device=device)
        work = _all_gather(recv, send, pg, world)
        pending.append((k, recv, work, send))
        # Bucket k-1's gather ran while bucket k was computed; apply it now so
        # only the last bucket's gather + apply remain after the compute.
        if len(pending) > 1:
            _apply_bucket(plan, pending.pop(0), apply)
    for item in pending:
        _apply_bucket(plan, item, apply)


def _apply_bucket(plan: ShardPlan, item, apply) -> None:
    k, recv, work, _send = item
    work.wait()
    size = plan.bucket_numel[k]
    for r in range(plan.world):
        base = r * size
        for i, off in plan.buckets[k][r]:
            n = numel(plan.shapes[i])
            apply(i, recv[base + off:base + off + n].view(plan.shapes[i]))


# --------------------------------------------------------------------------
# Owner apply + in-place parameter gather (collective="param_gather").
class ParamStore:
    """Per-bucket flat parameter storage laid out like the all-gather output.

    Bucket k holds ``world`` chunks of ``plan.bucket_numel[k]`` elements; rank
    r's chunk packs, at the plan's offsets, the parameters r owns in bucket
    k.  Every parameter's ``.data`` is re-pointed to a view of its slot (the
    current values are copied in first), so the Parameter objects the caller
    holds stay the same while their storage moves.  Then a step needs no
    receive buffer and no apply pass on non-owners: each owner updates its
    own parameters in place and one in-place all-gather per bucket delivers
    the new values straight into every rank's parameter storage.

    If a caller later replaces ``p.data`` (so the pointer leaves the slot),
    ``bind`` copies the new value back into the slot before the step.
    """

    def __init__(self, plan: ShardPlan, params, device):
        self.plan = plan
        self.dtype = params[0].dtype
        self.flats = [torch.zeros(plan.world * size, dtype=self.dtype, device=device)
                      for size in plan.bucket_numel]
        self.slots: list = [None] * len(params)
        for k, row in enumerate(plan.buckets):
            size = plan.bucket_numel[k]
            for r in range(plan.world):
                for i, off in row[r]:
                    base = r * size + off
                    self.slots[i] = self.flats[k][base:base + numel(plan.shapes[i])].view(
                        plan.shapes[i])
        self.bind(params)

    @staticmethod
    def supports(params) -> bool:
        """One dtype, one device, contiguous, and no parameter sharing storage
        with another (re-pointing would split a tied weight)."""
        if not params:
            return False
        dt, dev = params[0].dtype, params[0].device
        seen = set()
        for p in params:
            if p.dtype != dt or p.device != dev or not p.data.is_contiguous():
                return False
            key = p.data.untyped_storage().data_ptr()
            if key in seen:
                return False
            seen.add(key)
        return True

    def bind(self, params) -> None:
        for p, slot in zip(params, self.slots):
            if p.data.data_ptr() != slot.data_ptr():
                slot.copy_(p.data)
                p.data = slot


def _all_gather_inplace(flat: torch.Tensor, rank: int, pg, world: int):
    """All-gather whose input is this rank's own chunk of the output."""
    import torch.distributed as dist

    chunks = flat.chunk(world)
    if dist.get_backend(pg) == "nccl":
        return dist.all_gather_into_tensor(flat, chunks[rank], group=pg, async_op=True)
    return dist.all_gather(list(chunks), chunks[rank].clone(), group=pg, async_op=True)


def run_sharded_param_gather(store: ParamStore, rank: int, pg, compute, apply) -> None:
    """One sharded step with owner-side apply.

    For each bucket: ``compute(indices, out)`` writes the owned matrices'
    bf16 updates into a scratch buffer, ``apply(i, u)`` updates parameter i
    in place (it lives in this rank's chunk of the bucket's flat storage),
    then the bucket is all-gathered in place, asynchronously, so its
    transfer overlaps the next bucket's Newton-Schulz.  At the end the
    current stream waits for every gather, so later kernels on it (the next
    forward pass) read the new parameters.
    """
    plan = store.plan
    world = plan.world
    dev = store.flats[0].device if store.flats else None
    cap = max((plan.bucket_numel[k] for k in range(len(plan.buckets))), default=0)
    upd = torch.empty(max(cap, 1), dtype=torch.bfloat16, device=dev)
    works = []
    for k, row in enumerate(plan.buckets):
        if plan.bucket_numel[k] == 0:
            continue
        mine = row[rank]
        for idx, off0, n, shape in _runs(plan, mine):
            rows = shape[0]
            cols = numel(shape) // rows
            out = upd[off0:off0 + n * rows * cols].view(n, rows, cols)
            compute(idx, out)
            for j, i in enumerate(idx):
                apply(i, out[j])
        works.append(_all_gather_inplace(store.flats[k], rank, pg, world))
    for w in works:
        w.wait()


def _runs(plan: ShardPlan, mine):
    """Consecutive same-shape matrices of one rank's bucket share: one batched
    Newton-Schulz call each.  Yields (indices, offset, count, shape)."""
    j = 0
    while j < len(mine):
        i0, off0 = mine[j]
        shape = plan.shapes[i0]
        e = j + 1
        while e < len(mine) and plan.shapes[mine[e][0]] == shape:
            e += 1
        yield [i for i, _ in mine[j:e]], off0, e - j, shape
        j = e
