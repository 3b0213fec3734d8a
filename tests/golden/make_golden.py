"""Generate the golden vectors in this folder from the reference itself.

Runs only where a reference checkout exists: pass its path as the first
argument or in ``FUSED_MUON_REFERENCE``; the committed ``ns_golden.pt`` is what
the tests read, so nothing at test time needs the reference.

What is recorded (all on CPU, the reference's pure-PyTorch path):
* ``muon_fused/ns_step.py::_pytorch_newton_schulz`` outputs for small seeded
  inputs: wide, tall, square, ragged (non-multiple-of-8) shapes, fp32 and bf16
  inputs, steps in {0, 1, 5};
* the same function at BASELINE config 1, (896, 1152) N(0,1) seed 0, 5 steps,
  recorded as a SHA-256 of the output bytes plus summary values;
* one iteration as the reference's tests define it
  (tests/test_correctness.py:37-42) on a normalised (128, 192) input, seed 42;
* three steps of ``benchmarks/reference_muon.py::Muon`` (uncompiled NS, since
  the ``@torch.compile`` wrapper cannot build on a CPU-only box) on a small
  parameter set with ``use_muon`` and AdamW groups.

Usage: python tests/golden/make_golden.py <path to the reference checkout>
"""

from __future__ import annotations

import hashlib
import importlib.util
import os
import sys

import torch

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FUSED_MUON_REFERENCE", "")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ns_golden.pt")

NS_CASES = [
    # (rows, cols, seed, steps, dtype)
    (64, 96, 0, 5, "bf16"),
    (96, 64, 1, 5, "bf16"),
    (128, 128, 2, 5, "bf16"),
    (40, 72, 3, 5, "bf16"),
    (72, 40, 4, 5, "bf16"),
    (64, 80, 5, 5, "fp32"),
    (128, 192, 6, 1, "bf16"),
    (64, 96, 7, 0, "bf16"),
    (192, 256, 8, 5, "bf16"),
    (8, 200, 9, 5, "bf16"),
]


def _load(name: str, path: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def gen_input(rows: int, cols: int, seed: int, dtype: str) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    G = torch.randn(rows, cols, generator=g)
    return G.bfloat16() if dtype == "bf16" else G


def sha256(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def muon_params(seed: int = 11):
    g = torch.Generator().manual_seed(seed)
    shapes_muon = [(128, 64), (64, 128), (16, 8, 3)]
    shapes_adam = [(64,)]
    pm = [(torch.randn(s, generator=g) * 0.02) for s in shapes_muon]
    pa = [(torch.randn(s, generator=g) * 0.02) for s in shapes_adam]
    return pm, pa


def muon_grads(params, step: int):
    g = torch.Generator().manual_seed(1000 + step)
    return [torch.randn(p.shape, generator=g) * 1e-3 for p in params]


MUON_HP = dict(lr=0.02, wd=0.1, momentum=0.95, nesterov=True, ns_steps=5)
MUON_STEPS = 3


def main() -> None:
    if not REF or not os.path.isdir(REF):
        sys.exit("usage: make_golden.py <path to the reference checkout> "
                 "(or set FUSED_MUON_REFERENCE)")
    torch.set_num_threads(1)
    sys.path.insert(0, REF)
    ns = _load("ref_ns_step", os.path.join(REF, "muon_fused", "ns_step.py"))
    rm = _load("ref_reference_muon", os.path.join(REF, "benchmarks", "reference_muon.py"))
    plain_ns = rm.zeropower_via_newtonschulz5._torchdynamo_orig_callable
    rm.zeropower_via_newtonschulz5 = plain_ns  # Muon.step looks the name up at call time

    gold = {"ns": [], "meta": {"torch": str(torch.__version__), "threads": 1}}
    for rows, cols, seed, steps, dt in NS_CASES:
        G = gen_input(rows, cols, seed, dt)
        out = ns._pytorch_newton_schulz(G, steps)
        assert torch.equal(out, plain_ns(G, steps))
        gold["ns"].append(dict(rows=rows, cols=cols, seed=seed, steps=steps, dtype=dt, G=G.clone(), out=out.contiguous().clone()))

    G1 = gen_input(896, 1152, 0, "bf16")
    out1 = ns._pytorch_newton_schulz(G1, 5)
    gold["config1"] = dict(shape=(896, 1152), seed=0, steps=5, sha256_in=sha256(G1),
                           sha256_out=sha256(out1), norm=float(out1.float().norm()),
                           head=out1[0, :16].clone())

    g = torch.Generator().manual_seed(42)
    G = torch.randn(128, 192, generator=g).bfloat16()
    X = (G / (G.norm() + 1e-7)).contiguous()
    a, b, c = 3.4445, -4.7750, 2.0315
    A = X @ X.T
    B = b * A + c * A @ A
    gold["single_step"] = dict(X=X.clone(), out=(a * X + B @ X).contiguous().clone())

    pm, pa = muon_params()
    params = [p.clone() for p in pm + pa]
    groups = [dict(params=params[:3], use_muon=True), dict(params=params[3:], use_muon=False)]
    opt = rm.Muon(groups, **MUON_HP)
    for s in range(MUON_STEPS):
        for p, gr in zip(params, muon_grads(params, s)):
            p.grad = gr
        opt.step()
    gold["muon"] = dict(init=[p.clone() for p in pm + pa], hp=MUON_HP, steps=MUON_STEPS,
                        final=[p.detach().clone() for p in params],
                        momentum=[opt.state[p]["momentum_buffer"].clone() for p in params[:3]])
    torch.save(gold, OUT)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
