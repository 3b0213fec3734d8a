"""CUDA-graph capture of the front door and of the optimizer step.

Every entry point is asynchronous on the caller's stream with no host
synchronisation and no allocation after the first call for a shape, so a
caller can capture ``fused_newton_schulz`` or a whole ``FusedMuon.step()`` in
a CUDA graph (``torch.cuda.graph``) and replay it.  Tensor maps, the split-K
counter reset and the programmatic-dependent launches are all recorded in the
graph; a replay on new input data must equal an eager call bit for bit.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _randn(shape, seed, scale=1.0):
    return (torch.randn(shape, generator=torch.Generator().manual_seed(seed)) * scale)


@pytest.mark.parametrize("shape", [(1024, 2048), (1536, 768), (512, 2048), (300, 700),
                                   (2560, 3072)])
def test_ns_graph_replay_matches_eager(cuda_lib, shape):
    """Wide, tall (transposing path) and ragged shapes on the persistent kernel
    (a cooperative launch, captured like any other), and (2560, 3072) on the
    per-GEMM CTA-pair kernels."""
    from muon_fused import fused_newton_schulz, workspace_size

    G = _randn(shape, 0).bfloat16().to(DEV)
    ws = torch.empty(workspace_size(*shape), dtype=torch.uint8, device=DEV)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fused_newton_schulz(G, 5, ws)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = fused_newton_schulz(G, 5, ws)
    for seed in (1, 2):
        G.copy_(_randn(shape, seed).bfloat16())
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, fused_newton_schulz(G.clone(), 5)), seed


SHAPES = [(256, 512), (256, 512), (512, 256), (128, 64), (64, 32, 3, 3)]


def _params():
    return [torch.nn.Parameter((_randn(s, i, 0.02)).to(DEV)) for i, s in enumerate(SHAPES)]


def _grads(step):
    return [(_randn(s, 100 * step + i, 1e-3)).to(DEV) for i, s in enumerate(SHAPES)]


def test_optimizer_step_graph_replay_matches_eager(cuda_lib):
    """Four steps: eager, against one eager step followed by three replays of
    a captured step fed through static gradient tensors."""
    from muon_fused import FusedMuon

    eager = _params()
    opt_e = FusedMuon([{"params": eager, "use_muon": True}], lr=0.02)
    for st in range(4):
        for p, g in zip(eager, _grads(st)):
            p.grad = g
        opt_e.step()

    graphed = _params()
    opt_g = FusedMuon([{"params": graphed, "use_muon": True}], lr=0.02)
    static = _grads(0)
    for p, g in zip(graphed, static):
        p.grad = g
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        opt_g.step()  # step 0 runs eagerly: creates the state and the scratch arena
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        opt_g.step()  # recorded, not run
    for st in range(1, 4):
        for s, g in zip(static, _grads(st)):
            s.copy_(g)
        graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(eager, graphed):
        assert torch.equal(a.detach(), b.detach())
    for a, b in zip(eager, graphed):
        assert torch.equal(opt_e.state[a]["momentum_buffer"], opt_g.state[b]["momentum_buffer"])
