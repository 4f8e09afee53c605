"""The CPU oracle against golden vectors recorded from the reference itself.

Fixtures: tests/golden/scan.pt and tests/golden/mixer.pt, written by
tests/golden/make_golden.py from the reference's fast_scan.py (scan_eager,
autograd and manual_backward) and train_ablation.py (FastWeightMixer phases
1-3) in float64.
"""
import os

import pytest
import torch

import oracle

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(x, y):
    return (x - y).abs().max().item() / (y.abs().max().item() + 1e-30)


def _load(name):
    return torch.load(os.path.join(GOLD, name))["cases"]


SCAN = _load("scan.pt")
MIXER = _load("mixer.pt")


@pytest.mark.parametrize("case", SCAN, ids=[c["name"] for c in SCAN])
def test_scan_forward_matches_reference(case):
    ins = [case[k] for k in "U K a b m n".split()]
    S, M, V = oracle.scan_forward_all(*ins, case["rule"], case["ns"])
    assert rel(S, case["S"]) < 1e-12
    assert rel(M, case["M_all"]) < 1e-12 or case["rule"] == 0
    assert rel(V, case["V_all"]) < 1e-12 or case["rule"] != 2


@pytest.mark.parametrize("case", SCAN, ids=[c["name"] for c in SCAN])
def test_scan_backward_matches_reference_autograd(case):
    ins = [case[k] for k in "U K a b m n".split()]
    grads = oracle.scan_backward(*ins, case["S"], case["M_all"], case["V_all"], case["gS"],
                                 case["rule"], case["ns"])
    names = ["dU", "dK", "da", "db", "dm", "dn"]
    for name, g in zip(names, grads):
        ref = case[name]
        if ref.abs().max() == 0:
            # gates the rule never reads: the oracle must give exact zeros
            assert g.abs().max().item() == 0.0, name
        else:
            assert rel(g, ref) < 1e-10, name
    # the reference's own hand-derived VJP agrees too
    for name, g, man in zip(names, grads, case["manual"]):
        if case[name].abs().max() > 0:
            assert rel(g, man) < 1e-10, name


@pytest.mark.parametrize("case", SCAN[:4], ids=[c["name"] for c in SCAN[:4]])
def test_scan_autograd_of_oracle_matches(case):
    base = [case[k] for k in "U K a b m n".split()]
    ins = [t.clone().requires_grad_(True) for t in base]
    S = oracle.scan_forward(*ins, case["rule"], case["ns"])
    torch.autograd.backward(S, case["gS"])
    for t, name in zip(ins, ["dU", "dK", "da", "db", "dm", "dn"]):
        g = t.grad if t.grad is not None else torch.zeros_like(t)
        if case[name].abs().max() > 0:
            assert rel(g, case[name]) < 1e-10, name


def _mixer_inputs(case, requires_grad=False):
    names = ["q", "k", "v", "alpha", "beta", "mu", "nu"]
    ins = []
    for n in names:
        t = case[n]
        if t is not None:
            t = t.clone().requires_grad_(requires_grad)
        ins.append(t)
    return ins


@pytest.mark.parametrize("case", MIXER, ids=[c["name"] for c in MIXER])
def test_mixer_core_matches_reference(case):
    ins = _mixer_inputs(case, requires_grad=True)
    o = oracle.mixer_core_forward(*ins, case["rule"], case["ns"], case["chunk"])
    # the reference runs its phase 2 in fp32 even for fp64 activations
    # (train_ablation.py:170-181 cast the gate scalars and U/K with .float()),
    # so its fixtures carry fp32 rounding; the oracle here is fp64 throughout.
    assert rel(o, case["o"]) < 1e-5
    (o * case["dO"]).sum().backward()
    for t, name in zip(ins, ["dq", "dk", "dv", "dalpha", "dbeta", "dmu", "dnu"]):
        if t is None:
            continue
        ref = case[name]
        g = t.grad if t.grad is not None else torch.zeros_like(t)
        if ref.abs().max() == 0:
            assert g.abs().max().item() == 0.0, name
        else:
            assert rel(g, ref) < 1e-4, name


def _epilogue_cases():
    return torch.load(os.path.join(GOLD, "epilogue.pt"), weights_only=False)["cases"]


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-300)).item()


@pytest.mark.parametrize("case", _epilogue_cases(), ids=lambda c: c["name"])
def test_epilogue_matches_reference(case):
    """The per-head RMSNorm restatement against train_ablation.py:188-189 run on
    the reference module's own nn.RMSNorm: output, d_o and dweight."""
    tol = {torch.float64: 1e-12, torch.float32: 2e-6}.get(case["o"].dtype, 8e-3)
    o = case["o"].clone().requires_grad_(True)
    w = case["weight"].clone().requires_grad_(True)
    y = oracle.head_rmsnorm(o, w, None, case["out_dtype"])
    assert y.dtype == case["y"].dtype and y.shape == case["y"].shape
    assert _rel(y, case["y"]) <= tol
    (y.double() * case["dy"].double()).sum().backward()
    assert _rel(o.grad, case["d_o"]) <= tol
    assert _rel(w.grad, case["dweight"]) <= max(tol, 1e-5)


def _prologue_cases():
    return torch.load(os.path.join(GOLD, "prologue.pt"), weights_only=False)["cases"]


@pytest.mark.parametrize("case", _prologue_cases(), ids=lambda c: c["name"])
def test_prologue_matches_reference(case):
    """The prologue restatement against train_ablation.py:124-140 recorded in the
    reference module's own forward: q, k, v, gates and every input gradient."""
    tol = 1e-12 if case["u"].dtype == torch.float64 else 5e-6
    u = case["u"].clone().requires_grad_(True)
    gl = case["gl"].clone().requires_grad_(True)
    w = case["conv_w"].clone().requires_grad_(True)
    b = case["conv_b"].clone().requires_grad_(True)
    q, k, v, g = oracle.mixer_prologue(u, w, b, gl, case["n_heads"])
    for name, got in (("q", q), ("k", k), ("v", v), ("g", g)):
        assert _rel(got, case[name]) <= tol, name
    loss = sum((t * case["d" + n]).sum() for n, t in (("q", q), ("k", k), ("v", v), ("g", g)))
    loss.backward()
    for name, got in (("du", u.grad), ("dgl", gl.grad), ("dconv_w", w.grad), ("dconv_b", b.grad)):
        assert _rel(got, case[name]) <= max(tol, 2e-5), name
