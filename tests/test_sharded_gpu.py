"""Sharded FusedMuon over NCCL on 2 GPUs: every rank ends with parameters
bit-identical to a single-GPU run of the same optimizer (skipped with fewer
than 2 GPUs).  Ranks are child processes; NVLS is off (plain peer traffic)."""

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = [(1024, 512), (512, 1024), (768, 768), (256, 2048), (256, 2048), (2048, 256),
          (64, 32, 3, 3), (640, 640)]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _params(device):
    g = torch.Generator().manual_seed(0)
    return [torch.nn.Parameter((torch.randn(s, generator=g) * 0.02).to(device)) for s in SHAPES]


def _grads(step, device):
    g = torch.Generator().manual_seed(100 + step)
    return [(torch.randn(s, generator=g) * 1e-3).to(device) for s in SHAPES]


def _run(params, device, steps=3, collective="nccl"):
    from muon_fused import FusedMuon

    opt = FusedMuon([{"params": params, "use_muon": True}], lr=0.02, bucket_bytes=1 << 20,
                    collective=collective)
    for s in range(steps):
        for p, g in zip(params, _grads(s, device)):
            p.grad = g
        opt.step()
    opt.consolidate_state_dict()  # no-op on one process
    torch.cuda.synchronize(device)
    moms = [opt.state[p]["momentum_buffer"].cpu() for p in params]
    return [p.detach().cpu() for p in params], moms


def _worker(rank, world, port, outdir, collective):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        res = _run(_params(dev), dev, collective=collective)
        from muon_fused import _lib

        code = _lib.device_error()
        assert code == 0, f"rank {rank} ({collective}): device error code {code}"
        torch.save(res, os.path.join(outdir, f"{collective}{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_sharded_nccl_matches_single_gpu(cuda_lib):
    """Both exchanges (NCCL all-gather of the updates + apply on every rank;
    owner apply + in-place NCCL all-gather of the parameters) give every rank
    the same parameters, bit-identical between the two exchanges, and equal
    to the single-GPU run up to summation order.  After
    consolidate_state_dict() every rank holds every momentum buffer, equal to
    the single-GPU run's."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ref, ref_mom = _run(_params(torch.device("cuda", 0)), torch.device("cuda", 0))
    outdir = tempfile.mkdtemp()
    for collective in ("nccl", "param_gather"):
        mp.spawn(_worker, args=(2, _port(), outdir, collective), nprocs=2, join=True)
    from oracle import ns_oracle as O

    init = [p.detach().cpu() for p in _params("cpu")]
    got = {c: [torch.load(os.path.join(outdir, f"{c}{r}.pt")) for r in range(2)]
           for c in ("nccl", "param_gather")}
    for c in got:
        for a, b in zip(got[c][0][0], got[c][1][0]):
            assert torch.equal(a, b)  # every rank applied the same updates
        for r in range(2):
            # consolidated momentum state on every rank equals the single-GPU run's
            for a, b in zip(got[c][r][1], ref_mom):
                assert torch.equal(a, b)
    got = {c: [v[0] for v in got[c]] for c in got}
    for a, b in zip(got["nccl"][0], got["param_gather"][0]):
        assert torch.equal(a, b)  # same arithmetic, different transport
    # Batches differ between the sharded and the single-GPU run (so may the
    # K-splits): equal up to fp32 summation order inside the GEMMs.
    for a, b, p0 in zip(got["nccl"][0], ref, init):
        assert O.rel_fro(a - p0, b - p0) <= 5e-3
