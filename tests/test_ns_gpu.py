"""Parity of the sm_100a Newton-Schulz path against the CPU oracle.

Gates (tolerances are written in each test):
* relative Frobenius error <= 1e-2 against the algorithm in fp32
  (``oracle.ns_fp32``, or the same restatement run in fp32 on the GPU with
  TF32 off at sizes where the CPU would take minutes);
* max|Δ|/max|ref| < 0.05 against the reference's bf16 output, the reference's
  own gate (tests/test_correctness.py:96-105, 127-135);
* A and B bit-exactly symmetric (torch.equal with their transposes).
"""

import pytest
import torch

from oracle import ns_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _seeded(rows, cols, seed, dtype=torch.bfloat16):
    G = torch.randn(rows, cols, generator=torch.Generator().manual_seed(seed))
    return G.to(dtype)


def _ns(G, steps=5):
    from muon_fused import fused_newton_schulz

    out = fused_newton_schulz(G.to(DEV), steps)
    torch.cuda.synchronize()
    return out


def _fp32_gpu(G, steps=5):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return O.ns_fp32(G.to(DEV), steps)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_golden_cases(cuda_lib, golden):
    """Every reference golden vector: within 1e-2 of fp32 and inside the
    reference's own 5% max-relative gate of the reference's output."""
    for case in golden["ns"]:
        G, s = case["G"], case["steps"]
        out = _ns(G, s).cpu()
        assert out.dtype == torch.bfloat16 and out.shape == G.shape
        tag = (case["rows"], case["cols"], s, case["dtype"])
        assert O.rel_fro(out, O.ns_fp32(G, s)) <= 1e-2, tag
        assert O.max_rel(out, case["out"]) < 0.05, tag


def test_config1_896x1152(cuda_lib):
    """(896, 1152) N(0,1) seed 0, 5 steps."""
    G = _seeded(896, 1152, 0)
    out = _ns(G).cpu()
    ref = O.ns_reference_bf16(G, 5)
    assert O.rel_fro(out, O.ns_fp32(G, 5)) <= 1e-2
    assert O.max_rel(out, ref) < 0.05
    # and it tracks the kernels' CPU model closely (same roundings, different sum order)
    assert O.rel_fro(out, O.ns_b200_model(G, 5)) <= 8e-3


@pytest.mark.parametrize("shape", [(2048, 2048), (2048, 2560), (1024, 4096), (512, 2048)])
def test_against_cpu_fp32(cuda_lib, shape):
    G = _seeded(*shape, seed=1)
    out = _ns(G).cpu()
    assert O.rel_fro(out, O.ns_fp32(G, 5)) <= 1e-2


@pytest.mark.parametrize("shape", [(3584, 3584), (4096, 4096), (8192, 8192), (2560, 6144),
                                   (2560, 9728), (3584, 4608), (4096, 14336), (4096, 28672)])
def test_baseline_sweeps_fp32_gpu(cuda_lib, shape):
    """BASELINE configs 2 and 3 at full size, against the fp32 restatement on
    the GPU (TF32 off)."""
    G = torch.randn(*shape, generator=torch.Generator(device=DEV).manual_seed(0), device=DEV,
                    dtype=torch.bfloat16)
    out = _ns(G)
    assert O.rel_fro(out, _fp32_gpu(G)) <= 1e-2


@pytest.mark.parametrize("shape", [(2560, 2048), (9728, 2560), (72, 40), (1500, 1000)])
def test_tall_inputs(cuda_lib, shape):
    """Tall G goes through the transpose path (reference ns_step.py:41-54),
    untested by the reference's own suite."""
    G = _seeded(*shape, seed=2)
    out = _ns(G)
    assert out.shape == G.shape
    ref = _fp32_gpu(G)
    assert O.rel_fro(out, ref) <= 1e-2
    # same result as orthogonalising Gᵀ and transposing back (the norm's
    # summation order differs, so equal up to a few bf16 roundings)
    out_t = _ns(G.T.contiguous())
    assert O.rel_fro(out, out_t.T) <= 1e-2


@pytest.mark.parametrize("shape", [(40, 72), (100, 300), (1000, 1500), (129, 257), (8, 200),
                                   (1, 64), (300, 100)])
def test_ragged_shapes(cuda_lib, shape):
    """Shapes that are not multiples of the 128x256 tile, 64-wide K block or
    8-element row alignment (the reference falls back to PyTorch there,
    torch_binding.cu:75-88)."""
    G = _seeded(*shape, seed=3)
    out = _ns(G).cpu()
    assert O.rel_fro(out, O.ns_fp32(G, 5)) <= 1e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.float64])
def test_input_dtypes(cuda_lib, dtype):
    """Any floating input is cast to bf16 first (ns_step.py:40); output is bf16."""
    G = _seeded(256, 384, 4, dtype=dtype)
    out = _ns(G)
    assert out.dtype == torch.bfloat16
    ref_bf16_in = _ns(G.to(torch.bfloat16))
    assert torch.equal(out, ref_bf16_in)


def test_non_contiguous_input(cuda_lib):
    G = _seeded(512, 768, 5).to(DEV)
    view = G[:, ::2]  # column stride 2
    out = _ns(view)
    assert torch.equal(out, _ns(view.contiguous()))


@pytest.mark.parametrize("steps", [0, 1, 2, 7])
def test_step_counts(cuda_lib, steps):
    """The 1e-2 gate is stated for the 5-step call; bf16 rounding error grows
    by ~1.5e-3 per extra iteration (the CPU model gives 1.07e-2 at 7 steps,
    the reference's own bf16 path 3.6e-2), so 7 steps gets 1.5e-2."""
    G = _seeded(192, 320, 6)
    out = _ns(G, steps).cpu()
    tol = 1e-2 if steps <= 5 else 1.5e-2
    assert O.rel_fro(out, O.ns_fp32(G, steps)) <= tol


def test_deterministic(cuda_lib):
    G = _seeded(1024, 1536, 7).to(DEV)
    a, b = _ns(G), _ns(G)
    assert torch.equal(a, b)


def test_workspace_reuse(cuda_lib):
    from muon_fused import fused_newton_schulz, workspace_size

    G = _seeded(640, 896, 8).to(DEV)
    ws = torch.empty(workspace_size(640, 896), dtype=torch.bfloat16, device=DEV)
    a = fused_newton_schulz(G, 5, workspace=ws)
    b = fused_newton_schulz(G, 5, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(a, _ns(G))


def test_intermediates_bit_symmetric(cuda_lib):
    """A = X·Xᵀ and B are bit-exactly symmetric; A matches an fp32 product to
    bf16 rounding; B's off-diagonal and fp32 diagonal match the polynomial."""
    from muon_fused import _fused_muon_C as _C

    for shape in [(896, 1152), (2048, 2560), (300, 700)]:
        G = _seeded(*shape, seed=9).to(DEV)
        X = (G / (G.float().norm() + 1e-7)).to(torch.bfloat16).contiguous()
        A, B, d, X_new = _C.ns_step_debug(X)
        torch.cuda.synchronize()
        assert torch.equal(A, A.T), shape
        assert torch.equal(B, B.T), shape
        assert torch.count_nonzero(torch.diagonal(B)) == 0
        Xf = X.float()
        A32 = Xf @ Xf.T
        assert O.rel_fro(A, A32) <= 4e-3
        Af = A.float()
        P = O.C_COEF * (Af @ Af) + O.B_COEF * Af
        assert O.rel_fro(d, torch.diagonal(P) + O.A_COEF) <= 1e-5
        Poff = P - torch.diag(torch.diagonal(P))
        assert O.rel_fro(B, Poff) <= 4e-3


def test_single_step_reference_gate(cuda_lib, golden):
    """_C.newton_schulz_step against the reference's own single-step test
    (tests/test_correctness.py:78-105): max-relative error < 5%."""
    from muon_fused import _fused_muon_C as _C

    s = golden["single_step"]
    out = _C.newton_schulz_step(s["X"].to(DEV)).cpu()
    assert O.max_rel(out, s["out"]) < 0.05
    for shape in [(896, 896), (2048, 2048), (2048, 2560), (4096, 4096)]:
        torch.manual_seed(42)
        G = torch.randn(*shape, device=DEV, dtype=torch.bfloat16)
        X = (G / (G.norm() + 1e-7)).contiguous()
        fused = _C.newton_schulz_step(X)
        ref = O.ns_single_step_reference(X)
        assert O.max_rel(fused, ref) < 0.05, shape


def test_reference_multi_step_gate(cuda_lib):
    """The reference's multi-step test (tests/test_correctness.py:111-136) on
    its shapes: fused vs torch bf16 NS on the GPU, max-relative < 5%."""
    from muon_fused import _fused_muon_C as _C

    for shape in [(896, 896), (2048, 2048), (2048, 2560), (2560, 4096), (3584, 4608),
                  (4096, 4096)]:
        torch.manual_seed(123)
        G = torch.randn(*shape, device=DEV, dtype=torch.bfloat16)
        fused = _C.fused_newton_schulz(G, 5)
        ref = O.ns_reference_bf16(G, 5)
        assert fused.shape == G.shape
        assert O.max_rel(fused, ref) < 0.05, shape


def test_no_device_error(cuda_lib):
    from muon_fused import _lib

    _ns(_seeded(256, 512, 10))
    assert _lib.device_error() == 0


def test_orthogonality_property_full_size(cuda_lib):
    """Size-independent property at a full BASELINE size: for a wide Gaussian
    (n/m = 3.5, so sigma_min/sigma_max ~ 0.3) five quintic steps push every
    singular value into the band the reference documents
    (benchmarks/reference_muon.py:18-21: S' roughly in [0.5, 1.5]); the CPU
    model of the same arithmetic gives [0.68, 1.14] at (1024, 3584)."""
    G = torch.randn(4096, 14336, generator=torch.Generator(device=DEV).manual_seed(0), device=DEV,
                    dtype=torch.bfloat16)
    s = torch.linalg.svdvals(_ns(G).float())
    assert s.min() > 0.5 and s.max() < 1.3


@pytest.mark.parametrize("batch,rows,cols,kmax", [(64, 96, 128, 32), (4, 256, 1024, 8),
                                                  (3, 200, 72, 16)])
def test_normalisation_bit_exact(cuda_lib, batch, rows, cols, kmax):
    """steps=0 returns the normalised input bf16(bf16(G) / (||G||_F + 1e-7)).
    Entries k/32 with |k| <= kmax keep every partial sum of squares exact in
    fp32, so the denominator is known exactly and the output must equal an
    IEEE fp32 division rounded to bf16, element for element; this covers the
    kernels' reciprocal fast path and its exact-division fallback near bf16
    rounding midpoints."""
    from muon_fused import _fused_muon_C as _C

    g = torch.Generator().manual_seed(rows * cols + kmax)
    k = torch.randint(-kmax, kmax + 1, (batch, rows, cols), generator=g)
    G = (k.double() / 32).to(torch.bfloat16)
    out = _C.fused_newton_schulz_batched(G.to(DEV), 0).cpu()
    for b in range(batch):
        s = float((G[b].double() ** 2).sum())
        den = torch.sqrt(torch.tensor(s, dtype=torch.float32)) + 1e-7
        ref = (G[b].float() / den).to(torch.bfloat16)
        assert torch.equal(out[b], ref), b


@pytest.mark.parametrize("m,n", [(256, 384), (384, 448), (200, 440), (3072, 3072), (3072, 4096)])
def test_single_cta_and_pair_kernels_bit_identical(cuda_lib, m, n):
    """The single-CTA (128x256 tiles) and CTA-pair (256x256 tiles) kernels
    run the same per-element arithmetic: every output element is one fp32
    accumulation over K in the same K-block order, then the same epilogue.
    Where neither path splits K, one iteration gives bit-identical A, Boff,
    diag and X'.  The pair path splits K only when a GEMM has fewer than 74
    tiles and at least 8 K-blocks, so the shapes here have either K <= 448
    (short reductions) or m >= 3072 (78+ lower-triangle pair tiles).  With a
    K-split the fp32 partial sums are added in a different order and agree
    only to rounding (test_split_k_single_matrix)."""
    from muon_fused import _fused_muon_C as _C
    from muon_fused import _lib

    X = torch.randn(m, n, generator=torch.Generator().manual_seed(m + n)).bfloat16().to(DEV)
    X = (X.float() / X.float().norm()).bfloat16()
    res = {}
    try:
        for path in (1, 2):
            _lib.set_gemm_path(path)
            res[path] = _C.ns_step_debug(X)
    finally:
        _lib.set_gemm_path(0)
    torch.cuda.synchronize()
    for a, b, name in zip(res[1], res[2], ("A", "Boff", "diag", "X_new")):
        assert torch.equal(a, b), name
