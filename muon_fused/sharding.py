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


# --------------------------------------------------------------------------
# Peer-memory exchange: all-gather and apply fused into one kernel that reads
# each owner's send buffer over NVLink (fm_peer_gather_apply).
class _DevicePtr:
    """Zero-copy view of a library-owned device buffer (CUDA array interface)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes // 2,), "typestr": "<i2",
                                         "data": (ptr, False), "version": 3, "strides": None}


_ENTRY_DTYPE = None


def _entry_dtype():
    """numpy layout of fm_apply_entry (include/fused_muon.h)."""
    global _ENTRY_DTYPE
    if _ENTRY_DTYPE is None:
        import numpy as np

        _ENTRY_DTYPE = np.dtype([("param", "<u8"), ("numel", "<i8"), ("src_offset", "<i8"),
                                 ("decay", "<f4"), ("alpha", "<f4"), ("dtype", "<i4"),
                                 ("peer", "<i4")])
        assert _ENTRY_DTYPE.itemsize == 40
    return _ENTRY_DTYPE


class PeerExchange:
    """Double-buffered send buffers and per-bucket flags shared over CUDA IPC.

    Rank r owns a send buffer of 2 x share bf16 elements (step parity) and a
    flag array of 2 x buckets int64.  Every rank maps every other rank's
    buffers once (``all_gather_object`` of the IPC handles), so a step needs
    no collective call at all: owners raise ``flag[bucket] = step`` after the
    bucket's Newton-Schulz, readers wait on it inside the apply kernel.
    """

    def __init__(self, plan: ShardPlan, rank: int, pg, device):
        import ctypes

        import torch.distributed as dist

        from muon_fused import _lib

        lib = _lib.load()
        self.plan, self.rank, self.world = plan, rank, plan.world
        self.device = device
        self.nb = len(plan.buckets)
        self.bucket_off = []
        off = 0
        for k in range(self.nb):
            self.bucket_off.append(off)
            off += plan.bucket_numel[k]
        self.share = max(off, 1)
        self._own = []
        handles = []
        with torch.cuda.device(device):
            for nbytes in (2 * self.share * 2, 2 * self.nb * 8):
                ptr = ctypes.c_void_p()
                h = ctypes.create_string_buffer(64)
                _lib.check(lib.fm_peer_alloc(nbytes, ctypes.byref(ptr), h), "fm_peer_alloc")
                self._own.append(ptr.value)
                handles.append(h.raw)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, handles, group=pg)
        self._opened = []
        src, flags = [], []
        with torch.cuda.device(device):
            for r in range(self.world):
                if r == rank:
                    src.append(self._own[0])
                    flags.append(self._own[1])
                    continue
                ptrs = []
                for h in gathered[r]:
                    p = ctypes.c_void_p()
                    _lib.check(lib.fm_peer_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)),
                               "fm_peer_open")
                    ptrs.append(p.value)
                    self._opened.append(p.value)
                src.append(ptrs[0])
                flags.append(ptrs[1])
        self.peer_src = torch.tensor(src, dtype=torch.int64, device=device)
        self.peer_flags = torch.tensor(flags, dtype=torch.int64, device=device)
        self.send = torch.as_tensor(_DevicePtr(self._own[0], 2 * self.share * 2),
                                    device=device).view(torch.bfloat16)
        self.step = 0
        self._tables = None
        self._table_key = None

    def side_stream(self):
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(device=self.device)
        return self._side

    def bucket_view(self, k: int, parity: int) -> torch.Tensor:
        base = parity * self.share + self.bucket_off[k]
        return self.send[base:base + self.plan.bucket_numel[k]]

    def tables(self, params, decay_alpha):
        """Per-bucket device tables of fm_apply_entry, rebuilt when lr/wd change."""
        import numpy as np

        from muon_fused.optimizer import _EW_DTYPES

        key = (tuple(decay_alpha), tuple(p.data_ptr() for p in params))
        if self._table_key == key:
            return self._tables
        out = []
        for k, row in enumerate(self.plan.buckets):
            items = [(r, i, off) for r in range(self.world) for i, off in row[r]]
            arr = np.zeros(len(items), dtype=_entry_dtype())
            for j, (r, i, off) in enumerate(items):
                p = params[i].data
                arr[j] = (p.data_ptr(), p.numel(), self.bucket_off[k] + off, decay_alpha[i][0],
                          decay_alpha[i][1], _EW_DTYPES[p.dtype], r)
            t = torch.from_numpy(arr.view(np.uint8)).to(self.device)
            out.append((t, len(items)))
        self._tables, self._table_key = out, key
        return out

    def close(self):
        from muon_fused import _lib

        lib = _lib.load()
        for p in self._opened:
            lib.fm_peer_close(p)
        for p in self._own:
            lib.fm_peer_free(p)
        self._opened, self._own = [], []


def run_sharded_peer(ex: PeerExchange, params, decay_alpha, compute) -> None:
    """One sharded step over peer memory.  ``compute(indices, out)`` as in
    run_sharded.  Updates are applied by fm_peer_gather_apply on a side
    stream: bucket k's kernel (started once this rank's bucket k is done)
    waits on the GPU for every owner's flag of bucket k and reads over NVLink
    while later buckets are computed on the current stream.  The side stream first waits for the current stream (the
    parameters may still be read by earlier work) and the current stream
    waits for it at the end."""
    from muon_fused import _lib

    lib = _lib.load()
    plan, rank = ex.plan, ex.rank
    ex.step += 1
    parity = ex.step % 2
    cur = torch.cuda.current_stream(ex.device)
    stream = cur.cuda_stream
    side = ex.side_stream()
    side.wait_stream(cur)
    tables = ex.tables(params, decay_alpha)

    def apply(k):
        t, n = tables[k]
        _lib.check(lib.fm_peer_gather_apply(
            t.data_ptr(), n, ex.peer_src.data_ptr(), parity * ex.share, ex.peer_flags.data_ptr(),
            parity * ex.nb + k, ex.step, side.cuda_stream), "fm_peer_gather_apply")

    for k, row in enumerate(plan.buckets):
        send = ex.bucket_view(k, parity)
        mine = row[rank]
        j = 0
        while j < len(mine):
            i0, off0 = mine[j]
            shape = plan.shapes[i0]
            e = j + 1
            while e < len(mine) and plan.shapes[mine[e][0]] == shape:
                e += 1
            rows = shape[0]
            cols = numel(shape) // rows
            out = send[off0:off0 + (e - j) * rows * cols].view(e - j, rows, cols)
            compute([i for i, _ in mine[j:e]], out)
            j = e
        _lib.check(lib.fm_peer_signal(ex._own[1] + 8 * (parity * ex.nb + k), ex.step, stream),
                   "fm_peer_signal")
        # The apply of bucket k starts only after this rank's own bucket k is
        # done and signalled: then every rank raises flag k before any of its
        # apply blocks can sit on SMs waiting for others, so the waits cannot
        # form a cycle even where the blocks keep GEMM CTAs waiting.
        done = torch.cuda.Event()
        done.record(cur)
        side.wait_event(done)
        apply(k)
    cur.wait_stream(side)
