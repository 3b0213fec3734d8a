"""Matrix-sharded FusedMuon step on CPU gloo ranks (no GPU).

The Newton-Schulz call is replaced, in the child processes only, by the
oracle's fp32 restatement so the sharding logic (owner table, momentum
ownership, bucketed all-gather, apply order) runs without CUDA.  Checks:
identical parameters on every rank, equal to a single-process run; balanced
and deterministic owner tables; uneven shards; a rank that leaves between
steps surfaces as an error on the others; a consolidated checkpoint equals the
single-process state and resumes to the single-process trajectory.
"""

import copy
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from muon_fused.sharding import ShardPlan, ns_flops, numel


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


SHAPES = [(64, 32), (16, 64), (16, 64), (64, 64), (128, 32), (128, 32), (32, 128), (8, 4, 3, 3),
          (48, 40)]


def _make(seed=0):
    g = torch.Generator().manual_seed(seed)
    params = [torch.nn.Parameter(torch.randn(s, generator=g) * 0.02) for s in SHAPES]
    return params


def _grads(step):
    g = torch.Generator().manual_seed(500 + step)
    return [torch.randn(s, generator=g) * 1e-3 for s in SHAPES]


def _patch_ns():
    import muon_fused.optimizer as om
    from oracle import ns_oracle as O

    def ns_batched_cpu(G, steps, workspace, out):
        for b in range(G.shape[0]):
            out[b].copy_(O.ns_fp32(G[b].float(), steps).to(torch.bfloat16))
        return out

    om._ns_batched = ns_batched_cpu


def _run_steps(params, steps, bucket_bytes, collective="nccl"):
    from muon_fused import FusedMuon

    opt = FusedMuon([{"params": params, "use_muon": True}], lr=0.02, bucket_bytes=bucket_bytes,
                    collective=collective)
    for s in range(steps):
        for p, g in zip(params, _grads(s)):
            p.grad = g.clone()
        opt.step()
    return opt


def _worker(rank, world, port, outdir, bucket_bytes, leave_rank, collective="nccl"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=8))
    _patch_ns()
    params = _make()
    try:
        if leave_rank is not None and rank == leave_rank:
            # leaves between steps: no collective of this rank is in flight
            dist.destroy_process_group()
            return
        ids = [id(p) for p in params]
        if collective == "param_gather":
            from muon_fused import sharding

            def _no_fallback(*a, **k):
                raise AssertionError("param_gather step fell back to the update all-gather")

            sharding.run_sharded = _no_fallback  # every step must take the in-place exchange
        opt = _run_steps(params, 2, bucket_bytes, collective)
        assert [id(p) for p in opt.param_groups[0]["params"]] == ids  # same Parameter objects
        if collective == "param_gather":
            # the parameters still live in the store's flat buffers
            store = next(iter(opt._stores.values()))
            assert all(p.data_ptr() == s.data_ptr() for p, s in zip(params, store.slots))
        owned = sorted(i for i, p in enumerate(params) if "momentum_buffer" in opt.state[p])
        torch.save({"params": [p.detach().clone() for p in params], "owned": owned},
                   os.path.join(outdir, f"rank{rank}.pt"))
    except Exception as e:  # recorded for the parent to inspect
        with open(os.path.join(outdir, f"rank{rank}.err"), "w") as f:
            f.write(repr(e))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _spawn(world, bucket_bytes=1 << 30, leave_rank=None, collective="nccl"):
    outdir = tempfile.mkdtemp()
    mp.spawn(_worker, args=(world, _free_port(), outdir, bucket_bytes, leave_rank, collective),
             nprocs=world, join=True)
    return outdir


def _single_process():
    _patch_ns()
    params = _make()
    _run_steps(params, 2, 1 << 30)
    return [p.detach() for p in params]


def test_plan_assigns_each_matrix_once_and_balances():
    for world in (1, 2, 3, 4, 8):
        plan = ShardPlan.build(SHAPES, world, bucket_bytes=4096)
        assert sorted(plan.owner) == sorted(plan.owner) and len(plan.owner) == len(SHAPES)
        loads = [0.0] * world
        for i, r in enumerate(plan.owner):
            loads[r] += ns_flops(SHAPES[i])
        # LPT bound: no rank exceeds the average by more than the largest item
        assert max(loads) <= sum(loads) / world + max(ns_flops(s) for s in SHAPES) + 1e-6
        seen = set()
        for k, row in enumerate(plan.buckets):
            for r in range(world):
                end = 0
                for i, off in row[r]:
                    assert plan.owner[i] == r and i not in seen
                    assert off >= end  # non-overlapping packing
                    end = off + numel(SHAPES[i])
                    seen.add(i)
                assert end <= plan.bucket_numel[k]
        assert seen == set(range(len(SHAPES)))
        # deterministic: the same shapes give the same table on every rank
        assert ShardPlan.build(SHAPES, world, 4096).owner == plan.owner


def test_plan_8b_shapes_balance():
    """the 224 matrices of the 8B set over 2/4/8 ranks."""
    per_layer = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096),
                 (14336, 4096), (4096, 14336)]
    shapes = per_layer * 32
    total = sum(ns_flops(s) for s in shapes)
    for world in (2, 4, 8):
        plan = ShardPlan.build(shapes, world)
        loads = [0.0] * world
        for i, r in enumerate(plan.owner):
            loads[r] += ns_flops(shapes[i])
        assert max(loads) / (total / world) < 1.03


@pytest.mark.parametrize("world,collective", [(2, "nccl"), (4, "nccl"), (2, "param_gather"),
                                               (4, "param_gather")])
def test_sharded_equals_single_process(world, collective):
    """Both exchanges: the update all-gather + apply everywhere, and the
    owner apply + in-place parameter all-gather (non-owners apply nothing)."""
    ref = _single_process()
    # small buckets: several all-gathers
    outdir = _spawn(world, bucket_bytes=8192, collective=collective)
    results = [torch.load(os.path.join(outdir, f"rank{r}.pt")) for r in range(world)]
    owned = []
    for r, res in enumerate(results):
        for a, b in zip(res["params"], ref):
            assert torch.equal(a, b)
        owned += res["owned"]
    # momentum state lives only on the owner rank: every matrix exactly once
    assert sorted(owned) == list(range(len(SHAPES)))


def test_rank_leaving_between_steps_is_an_error():
    outdir = _spawn(2, leave_rank=1)
    assert not os.path.exists(os.path.join(outdir, "rank0.pt"))
    with open(os.path.join(outdir, "rank0.err")) as f:
        assert f.read()


def test_param_store_repoints_and_rebinds():
    """ParamStore moves each parameter into its bucket slot (same Parameter
    object, same values) and copies a replaced ``.data`` back into the slot."""
    from muon_fused.sharding import ParamStore

    params = _make()
    before = [p.detach().clone() for p in params]
    plan = ShardPlan.build([tuple(p.shape) for p in params], 3, bucket_bytes=4096)
    store = ParamStore(plan, params, torch.device("cpu"))
    for p, b, slot in zip(params, before, store.slots):
        assert p.data_ptr() == slot.data_ptr() and torch.equal(p.detach(), b)
    params[2].data = torch.full_like(params[2].data, 7.0)
    store.bind(params)
    assert params[2].data_ptr() == store.slots[2].data_ptr()
    assert torch.all(store.slots[2] == 7.0)
    # tied weights (shared storage) are not supported: the plain exchange is used
    assert not ParamStore.supports([params[0], params[0]])


def _ckpt_worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    from muon_fused import FusedMuon

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    _patch_ns()
    try:
        params = _make()
        opt = _run_steps(params, 2, 8192)
        opt.consolidate_state_dict()
        sd = copy.deepcopy(opt.state_dict())  # as saved to disk: no tensors shared with opt
        # resume: a fresh sharded optimizer loads the checkpoint, runs step 3
        opt2 = FusedMuon([{"params": params, "use_muon": True}], lr=0.02, bucket_bytes=8192)
        opt2.load_state_dict(copy.deepcopy(sd))  # load_state_dict keeps the given tensors
        for p, g in zip(params, _grads(2)):
            p.grad = g.clone()
        opt2.step()
        kept = sorted(i for i, p in enumerate(params) if "momentum_buffer" in opt2.state[p])
        torch.save({"state": sd["state"], "params": [p.detach() for p in params], "kept": kept},
                   os.path.join(outdir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_consolidated_checkpoint_matches_single_process_and_resumes(world):
    _patch_ns()
    params = _make()
    opt = _run_steps(params, 2, 1 << 30)
    ref_state = copy.deepcopy(opt.state_dict()["state"])  # step 3 below updates buffers in place
    for p, g in zip(params, _grads(2)):
        p.grad = g.clone()
    opt.step()
    ref_params = [p.detach() for p in params]
    outdir = tempfile.mkdtemp()
    mp.spawn(_ckpt_worker, args=(world, _free_port(), outdir), nprocs=world, join=True)
    kept = []
    for r in range(world):
        res = torch.load(os.path.join(outdir, f"rank{r}.pt"))
        # every rank's consolidated state has every buffer, equal to one process's
        assert sorted(res["state"]) == sorted(ref_state)
        for k, v in ref_state.items():
            assert torch.equal(res["state"][k]["momentum_buffer"], v["momentum_buffer"])
        for a, b in zip(res["params"], ref_params):
            assert torch.equal(a, b)
        kept += res["kept"]
    # after the resumed step each buffer is kept by its owner only
    assert sorted(kept) == list(range(len(SHAPES)))
