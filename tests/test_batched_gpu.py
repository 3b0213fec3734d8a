"""Batched Newton-Schulz and split-K scheduling.

One batched call (fm_fused_newton_schulz_batched) must give, per matrix, the
result of the single-matrix call up to fp32 summation order (the batch and
the single call may pick different K-splits), stay within the 1e-2 fp32 gate,
and be deterministic run to run (split-K partials are summed in split order,
not arrival order).
"""

import pytest
import torch

from oracle import ns_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _batch(b, rows, cols, seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(b, rows, cols, generator=g).to(dtype)


@pytest.mark.parametrize("b,rows,cols", [(8, 512, 2048), (3, 1152, 896), (5, 100, 300),
                                         (4, 2048, 2048), (2, 896, 1152), (16, 256, 512)])
def test_batched_matches_single_and_fp32(cuda_lib, b, rows, cols):
    from muon_fused import _fused_muon_C as _C

    G = _batch(b, rows, cols, seed=rows + cols)
    out = _C.fused_newton_schulz_batched(G.to(DEV), 5)
    torch.cuda.synchronize()
    assert out.shape == G.shape and out.dtype == torch.bfloat16
    for i in range(b):
        single = _C.fused_newton_schulz(G[i].to(DEV), 5)
        # same arithmetic up to the K-split (fp32 summation order)
        assert O.rel_fro(out[i], single) <= 5e-3, i
        if rows * cols <= 1 << 20:
            assert O.rel_fro(out[i].cpu(), O.ns_fp32(G[i], 5)) <= 1e-2, i


def test_batched_deterministic_and_strided_input(cuda_lib):
    from muon_fused import _fused_muon_C as _C

    big = _batch(6, 640, 1536, seed=11).to(DEV)
    a = _C.fused_newton_schulz_batched(big, 5)
    b = _C.fused_newton_schulz_batched(big, 5)
    assert torch.equal(a, b)
    # every other matrix of the batch: matrix stride 2x, same row stride
    sub = big[::2]
    c = _C.fused_newton_schulz_batched(sub, 5)
    d = _C.fused_newton_schulz_batched(sub.contiguous(), 5)
    assert torch.equal(c, d)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_batched_dtypes(cuda_lib, dtype):
    from muon_fused import _fused_muon_C as _C

    G = _batch(3, 384, 768, seed=5, dtype=dtype).to(DEV)
    assert torch.equal(_C.fused_newton_schulz_batched(G, 5),
                       _C.fused_newton_schulz_batched(G.to(torch.bfloat16), 5))


@pytest.mark.parametrize("shape", [(512, 2048), (1024, 4096), (2048, 2048), (300, 700)])
def test_split_k_single_matrix(cuda_lib, shape):
    """Shapes whose tile count is below the 74 CTA pairs run split-K; the
    result is deterministic and within the fp32 gate, and the single-CTA
    path (no split) agrees to summation order."""
    from muon_fused import _fused_muon_C as _C
    from muon_fused import _lib

    G = torch.randn(*shape, generator=torch.Generator().manual_seed(9)).bfloat16()
    Gd = G.to(DEV)
    a = _C.fused_newton_schulz(Gd, 5)
    b = _C.fused_newton_schulz(Gd, 5)
    assert torch.equal(a, b)
    try:
        _lib.set_gemm_path(1)
        c = _C.fused_newton_schulz(Gd, 5)
    finally:
        _lib.set_gemm_path(0)
    torch.cuda.synchronize()
    assert O.rel_fro(a, c) <= 5e-3
    if shape[0] * shape[1] <= 1 << 21:
        assert O.rel_fro(a.cpu(), O.ns_fp32(G, 5)) <= 1e-2
    assert _lib.device_error() == 0


def _set_shapes():
    """Distinct Muon matrix shapes of the 1B and 8B sets (BASELINE configs 4
    and 5) with their counts: q/o, k/v, gate/up, down per layer."""
    out = []
    for h, kv, ffn, layers in ((2048, 512, 8192, 16), (4096, 1024, 14336, 32)):
        out += [((h, h), 2 * layers), ((kv, h), 2 * layers), ((ffn, h), 2 * layers),
                ((h, ffn), layers)]
    return out


@pytest.mark.parametrize("shape,count", _set_shapes(),
                         ids=[f"{s[0]}x{s[1]}" for s, _ in _set_shapes()])
def test_optimizer_batches_full_size(cuda_lib, shape, count):
    """One batched call per distinct 1B/8B shape at the batch size FusedMuon
    forms for it (FusedMuon._batch_limit under the default 4 GiB budget,
    capped by the matrices of that shape in the set), tall gate/up shapes
    included.  A sample of each batch (first, middle, last matrix) is gated
    against the fp32 restatement on the GPU with TF32 off, <= 1e-2."""
    from muon_fused import FusedMuon
    from muon_fused import _fused_muon_C as _C

    rows, cols = shape
    opt = FusedMuon([torch.nn.Parameter(torch.zeros(1, device=DEV))])
    b = min(count, opt._batch_limit(rows, cols))
    gen = torch.Generator(device=DEV).manual_seed(rows * 7 + cols)
    G = (torch.randn(b, rows, cols, generator=gen, device=DEV) * 1e-3).bfloat16()
    out = _C.fused_newton_schulz_batched(G, 5)
    torch.cuda.synchronize()
    assert out.shape == G.shape
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for i in sorted({0, b // 2, b - 1}):
            ref = O.ns_fp32(G[i], 5)
            assert O.rel_fro(out[i], ref) <= 1e-2, (shape, b, i)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    from muon_fused import _lib

    assert _lib.device_error() == 0
