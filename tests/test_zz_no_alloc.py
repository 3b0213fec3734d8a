"""fm_fused_newton_schulz_noalloc: the allocation-free entry point.

Some callers cannot allocate device memory while they run: a host framework
that owns every byte of device memory through its own pool, or a step where a
cudaMalloc could stall or fail.  For them the library offers a Newton-Schulz
call whose scratch lives in a fixed device array inside the library.  This
test calls it through the C ABI, twice in a row on different inputs (the
array keeps the previous call's contents), and checks each result against the
regular entry point with a caller-allocated workspace.  Both run the same
plan and the same arithmetic, so the gate is bit equality (tighter than the
1e-2 relative-Frobenius tolerance against fp32 that the other parity tests
use, which is checked too).  It also checks that a call leaves the device's
free memory unchanged (the library allocates nothing behind torch's back) and
that an oversized matrix is refused with a clear error.

The file name sorts last so that a run stopping at the first failure has run
every other test already; it passes alone and after the others.
"""

import pytest
import torch

from oracle import ns_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _regular(lib, G, steps):
    from muon_fused import _lib

    out = torch.empty(G.shape, dtype=torch.bfloat16, device=DEV)
    need = _lib.workspace_bytes(*G.shape)
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    rc = lib.fm_fused_newton_schulz(G.data_ptr(), _lib.FM_DT_BF16, G.shape[0], G.shape[1],
                                    G.stride(0), out.data_ptr(), steps, ws.data_ptr(), need,
                                    torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "fm_fused_newton_schulz")
    return out


def _noalloc(lib, G, steps, out=None):
    from muon_fused import _lib

    if out is None:
        out = torch.empty(G.shape, dtype=torch.bfloat16, device=DEV)
    rc = lib.fm_fused_newton_schulz_noalloc(G.data_ptr(), _lib.FM_DT_BF16, G.shape[0],
                                            G.shape[1], G.stride(0), out.data_ptr(), steps,
                                            torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "fm_fused_newton_schulz_noalloc")
    return out


def test_noalloc_matches_regular_entry_point(cuda_lib):
    from muon_fused import _lib

    cases = [((1024, 1536), 0), ((1152, 896), 1)]  # wide, then tall (transpose path)
    for (rows, cols), seed in cases:
        G = torch.randn(rows, cols, generator=torch.Generator().manual_seed(seed)).bfloat16()
        Gd = G.to(DEV)
        got = _noalloc(cuda_lib, Gd, 5)
        want = _regular(cuda_lib, Gd, 5)
        torch.cuda.synchronize()
        assert got.shape == G.shape and got.dtype == torch.bfloat16
        assert torch.equal(got, want), (rows, cols)
        assert O.rel_fro(got.cpu(), O.ns_fp32(G, 5)) <= 1e-2, (rows, cols)
    assert _lib.device_error() == 0


def test_noalloc_allocates_no_device_memory(cuda_lib):
    """After a warm-up call (which may load the module and look up the
    array's address), a further call on a fresh input leaves the device's
    free memory exactly as it was."""
    G0 = torch.randn(1024, 2048, generator=torch.Generator().manual_seed(3)).bfloat16().to(DEV)
    G1 = torch.randn(1024, 2048, generator=torch.Generator().manual_seed(4)).bfloat16().to(DEV)
    out = torch.empty(G1.shape, dtype=torch.bfloat16, device=DEV)
    _noalloc(cuda_lib, G0, 5)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    _noalloc(cuda_lib, G1, 5, out=out)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.equal(out, _regular(cuda_lib, G1, 5))


def test_noalloc_rejects_oversized(cuda_lib):
    from muon_fused import _lib

    G = torch.empty(4096, 4096, dtype=torch.bfloat16, device=DEV)
    out = torch.empty_like(G)
    rc = cuda_lib.fm_fused_newton_schulz_noalloc(G.data_ptr(), _lib.FM_DT_BF16, 4096, 4096, 4096,
                                                 out.data_ptr(), 5,
                                                 torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.FM_E_WORKSPACE
    assert b"scratch" in cuda_lib.fm_last_error()
