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
   gathered buffers.

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
        j = 0
        while j < len(mine):
            # a run of consecutive same-shape matrices is one batched call
            i0, off0 = mine[j]
            shape = plan.shapes[i0]
            e = j + 1
            while e < len(mine) and plan.shapes[mine[e][0]] == shape:
                e += 1
            rows = shape[0]
            cols = numel(shape) // rows
            n = e - j
            out = send[off0:off0 + n * rows * cols].view(n, rows, cols)
            compute([i for i, _ in mine[j:e]], out)
            j = e
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
