"""The CPU oracle reproduces the reference's own outputs bit for bit
(golden vectors recorded by tests/golden/make_golden.py from the reference)."""

import hashlib

import pytest
import torch

from oracle import ns_oracle as O


def _sha(t):
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


@pytest.fixture(autouse=True)
def _one_thread():
    n = torch.get_num_threads()
    torch.set_num_threads(1)  # the goldens were recorded single-threaded
    yield
    torch.set_num_threads(n)


def test_ns_reference_matches_golden(golden):
    for case in golden["ns"]:
        out = O.ns_reference_bf16(case["G"], case["steps"])
        assert out.shape == case["out"].shape
        assert out.dtype == torch.bfloat16
        assert torch.equal(out, case["out"]), (case["rows"], case["cols"], case["steps"])


def test_config1_hash(golden):
    c = golden["config1"]
    G = torch.randn(*c["shape"], generator=torch.Generator().manual_seed(c["seed"])).bfloat16()
    assert _sha(G) == c["sha256_in"]
    out = O.ns_reference_bf16(G, c["steps"])
    assert _sha(out) == c["sha256_out"]
    assert torch.equal(out[0, :16], c["head"])


def test_single_step_matches_golden(golden):
    s = golden["single_step"]
    assert torch.equal(O.ns_single_step_reference(s["X"]), s["out"])


def test_muon_reference_step_matches_golden(golden):
    g = golden["muon"]
    params = [p.clone() for p in g["init"]]
    hp = g["hp"]
    groups = [
        dict(params=params[:3], use_muon=True, lr=hp["lr"], wd=hp["wd"], momentum=hp["momentum"],
             nesterov=hp["nesterov"], ns_steps=hp["ns_steps"]),
        dict(params=params[3:], use_muon=False, lr=hp["lr"], wd=hp["wd"],
             adamw_betas=(0.9, 0.95), adamw_eps=1e-8),
    ]
    state = {}
    from tests.golden.make_golden import muon_grads

    for s in range(g["steps"]):
        for p, gr in zip(params, muon_grads(params, s)):
            p.grad = gr
        O.muon_reference_step(groups, state)
    for p, f in zip(params, g["final"]):
        assert torch.equal(p, f)
    for p, mb in zip(params[:3], g["momentum"]):
        assert torch.equal(state[id(p)]["momentum_buffer"], mb)


def test_b200_model_accuracy(golden):
    """The kernels' arithmetic (bf16 storage, fp32 epilogues, fp32 diagonal of
    B) stays within the 1e-2 relative-Frobenius gate of an fp32 NS on every
    golden case, and within the reference's own max-relative gate (0.05,
    reference tests/test_correctness.py:127-135) of the reference's output."""
    for case in golden["ns"]:
        G, s = case["G"], case["steps"]
        model = O.ns_b200_model(G, s)
        assert O.rel_fro(model, O.ns_fp32(G, s)) <= 1e-2
        assert O.max_rel(model, case["out"]) < 0.05


def test_transpose_rule():
    """Tall inputs are orthogonalised through the transpose (ns_step.py:41-54)."""
    G = torch.randn(48, 16, generator=torch.Generator().manual_seed(3))
    a = O.ns_fp32(G, 3)
    b = O.ns_fp32(G.T.contiguous(), 3).T
    assert torch.allclose(a, b, atol=1e-6)
