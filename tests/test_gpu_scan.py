"""GPU parity of the phase-2 state scan against the CPU oracle.

Mirrors the reference's own check (test.py:41-68: eager vs kernel, every rule,
ns 3 and 5, forward states and every input gradient, on the realistic PSD
fixture of test.py:28-38), and extends it to other head dims, chunk counts,
gate ranges, ns = 0, the golden fixtures recorded from the reference, and the
full config-1 size through per-(b,h) slices.
"""
import os

import pytest
import torch

import oracle
from conftest import load_pkg
from oracle_runs import scan_oracle
from parity import TOL_FP32, check_outputs, perturb, rel

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NAMES = ["dU", "dK", "da", "db", "dm", "dn"]


def run_kernel(pkg, base, gS, rule, ns, precision):
    ins = [t.detach().float().cuda().requires_grad_(True) for t in base]
    S = pkg.state_scan(*ins, rule, ns, precision)
    S.backward(gS.float().cuda())
    torch.cuda.synchronize()
    return S.detach().cpu(), [t.grad.detach().cpu() for t in ins]


def scan_ref_fn(base, gS, rule, ns, gold=None):
    """ref_fn for parity.check_outputs; `gold` replaces the fp64 evaluation."""
    def fn(dtype, seed):
        if dtype == torch.float64 and gold is not None:
            return gold
        ins = base if seed is None else [perturb(t.float(), seed) for t in base]
        S, g = scan_oracle(ins, gS, rule, ns, dtype)
        return dict(zip(["S"] + NAMES, [S] + g))
    return fn


def compare(pkg, base, rule, ns, precision, tol, seed=7):
    gS = torch.randn(base[0].shape, generator=torch.Generator().manual_seed(seed))
    S, g = run_kernel(pkg, base, gS, rule, ns, precision)
    check_outputs(dict(zip(["S"] + NAMES, [S] + g)), scan_ref_fn(base, gS, rule, ns), tol,
                  widen=(tol == TOL_FP32 and rule != 0))


@pytest.mark.parametrize("rule,ns", [(0, 3), (0, 5), (1, 3), (1, 5), (2, 3), (2, 5)])
def test_reference_fixture_ieee(rule, ns):
    """test.py part 1: B4 H12 N16 C64 dh64, ieee precision."""
    pkg = load_pkg()
    base = pkg.workloads.scan_inputs(4, 12, 16, 64, C=64, seed=rule * 10 + ns)
    compare(pkg, base, rule, ns, pkg.GMDN_PREC_IEEE, TOL_FP32)


@pytest.mark.parametrize("dh", [16, 32, 128])
@pytest.mark.parametrize("rule,ns", [(0, 3), (1, 0), (1, 5), (2, 3)])
@pytest.mark.parametrize("N", [1, 2, 9])
def test_shapes_ieee(dh, rule, ns, N):
    pkg = load_pkg()
    base = pkg.workloads.scan_inputs(2, 3, N, dh, C=64, seed=100 + dh + N)
    compare(pkg, base, rule, ns, pkg.GMDN_PREC_IEEE, TOL_FP32)


@pytest.mark.parametrize("rule,ns", [(0, 3), (1, 5), (2, 3)])
def test_wide_gates_ieee(rule, ns):
    pkg = load_pkg()
    base = pkg.workloads.scan_inputs(1, 4, 12, 64, C=64, seed=300 + rule, family="wide")
    compare(pkg, base, rule, ns, pkg.GMDN_PREC_IEEE, TOL_FP32)


@pytest.mark.parametrize("rule,ns", [(0, 3), (1, 5), (2, 3)])
def test_fast_precision(rule, ns):
    """set_precision('tf32') equivalent; bound of the reference's own tf32 check
    (test.py:74 compares at 5e-2)."""
    pkg = load_pkg()
    base = pkg.workloads.scan_inputs(2, 4, 16, 128, C=64, seed=400 + rule)
    compare(pkg, base, rule, ns, pkg.GMDN_PREC_FAST, 5e-2)


def test_golden_fixtures():
    """The reference's own float64 outputs (tests/golden/scan.pt)."""
    pkg = load_pkg()
    for case in torch.load(os.path.join(GOLD, "scan.pt"))["cases"]:
        base = [case[k] for k in "U K a b m n".split()]
        S, g = run_kernel(pkg, base, case["gS"], case["rule"], case["ns"], pkg.GMDN_PREC_IEEE)
        gold = {n: case[n] for n in ["S"] + NAMES}
        check_outputs(dict(zip(["S"] + NAMES, [S] + g)),
                      scan_ref_fn(base, case["gS"], case["rule"], case["ns"], gold), TOL_FP32,
                      prefix=case["name"] + ":", widen=case["rule"] != 0)


def test_unused_gate_gradients_are_zero():
    """The reference's Triton backward returns torch.empty_like garbage for
    db/dm (delta) and dn (muon) (fast_scan.py:386-389); these must be zeros."""
    pkg = load_pkg()
    base = pkg.workloads.scan_inputs(2, 2, 4, 32, seed=5)
    for rule, zero in ((0, ["db", "dm", "dn"]), (1, ["dn"])):
        gS = torch.randn(base[0].shape)
        _, g = run_kernel(pkg, base, gS, rule, 3, pkg.GMDN_PREC_IEEE)
        for name in zero:
            assert g[NAMES.index(name)].abs().max().item() == 0.0, (rule, name)


@pytest.mark.parametrize("rule,ns", [(0, 3), (2, 3), (1, 5)])
def test_full_size_slices(rule, ns):
    """Config-1 scan size (B8 H16 N64 dh128): every (b,h) is independent, so a
    slice of the full run must equal the oracle on that slice and, bit for bit,
    the kernel run on that slice alone."""
    pkg = load_pkg()
    B, H, N, dh = 8, 16, 64, 128
    base = pkg.workloads.scan_inputs(B, H, N, dh, C=64, seed=11 + rule)
    gS = torch.randn(base[0].shape, generator=torch.Generator().manual_seed(3))
    S, g = run_kernel(pkg, base, gS, rule, ns, pkg.GMDN_PREC_IEEE)
    for (b, h) in ((0, 0), (5, 9), (7, 15)):
        sl = [t[b:b + 1, h:h + 1] for t in base]
        gsl = gS[b:b + 1, h:h + 1]
        got = dict(zip(["S"] + NAMES, [S[b:b + 1, h:h + 1]] + [a[b:b + 1, h:h + 1] for a in g]))
        check_outputs(got, scan_ref_fn(sl, gsl, rule, ns), TOL_FP32, prefix=f"({b},{h}):",
                      widen=rule != 0)
        S1, g1 = run_kernel(pkg, sl, gsl, rule, ns, pkg.GMDN_PREC_IEEE)
        assert torch.equal(S1, S[b:b + 1, h:h + 1])
        for a, a1 in zip(g, g1):
            assert torch.equal(a1, a[b:b + 1, h:h + 1])


def test_shim_matches_op():
    pkg = load_pkg()
    fs = pkg.fast_scan
    base = pkg.workloads.scan_inputs(1, 2, 4, 64, seed=9)
    fs.set_precision("ieee")
    S_shim = fs.fast_state_scan(*[t.cuda() for t in base], 2, 3).cpu()
    S_cls = fs._TritonScan.apply(*[t.cuda() for t in base], 2, 3).cpu()
    S_op = pkg.state_scan(*[t.cuda() for t in base], 2, 3, pkg.GMDN_PREC_IEEE).cpu()
    fs.set_precision("tf32")
    assert torch.equal(S_shim, S_op) and torch.equal(S_cls, S_op)
    S64 = oracle.scan_forward(*[t.double() for t in base], 2, 3)
    assert rel(S_op, S64) < 1e-4


def test_empty_chunk_axis():
    pkg = load_pkg()
    U = torch.zeros(2, 3, 0, 16, 16, device="cuda")
    g = torch.zeros(2, 3, 0, device="cuda")
    S = pkg.state_scan(U, U, g, g, g, g, 1, 3)
    assert S.shape == (2, 3, 0, 16, 16)


def _launched(pkg, fn):
    L = pkg._lib
    L.prof_report()
    L.prof_enable(True)
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        L.prof_enable(False)
    return set(L.prof_report())


@pytest.mark.parametrize("rule,ns", [(0, 3)])
@pytest.mark.parametrize("N", [1, 2, 9, 64])
def test_tensor_core_scan(rule, N, ns):
    """GMDN_PREC_FAST at dh 128, delta: the forward runs scan_fwd_tc, the
    split-bf16 tcgen05 scan, and the backward its reverse chain and the dK / da
    kernel on the tensor cores; states and every gradient against the oracle
    at the fp32 bar, on the reference fixture's input family (test.py:28-38)."""
    pkg = load_pkg()
    base = pkg.workloads.scan_inputs(2, 3, N, 128, C=64, seed=500 + 10 * rule + N)
    gS = torch.randn(base[0].shape, generator=torch.Generator().manual_seed(5))
    names = _launched(pkg, lambda: run_kernel(pkg, base, gS, rule, ns, pkg.GMDN_PREC_FAST))
    assert "scan_fwd_tc" in names, names
    if rule == 0:
        assert {"scan_bwd_chain_tc", "scan_bwd_dk_tc"} <= names, names
    S, g = run_kernel(pkg, base, gS, rule, ns, pkg.GMDN_PREC_FAST)
    check_outputs(dict(zip(["S"] + NAMES, [S] + g)), scan_ref_fn(base, gS, rule, ns), TOL_FP32,
                  widen=rule != 0)


@pytest.mark.parametrize("rule,ns", [(0, 3)])
def test_tensor_core_scan_config1_slices(rule, ns):
    """Config-1 scan size (B8 H16 N64 dh128) on the tensor-core scan: slices
    against the oracle on the same slice."""
    pkg = load_pkg()
    B, H, N, dh = 8, 16, 64, 128
    base = pkg.workloads.scan_inputs(B, H, N, dh, C=64, seed=21 + rule)
    gS = torch.randn(base[0].shape, generator=torch.Generator().manual_seed(4))
    S, g = run_kernel(pkg, base, gS, rule, ns, pkg.GMDN_PREC_FAST)
    for (b, h) in ((0, 0), (7, 15)):
        sl = [t[b:b + 1, h:h + 1] for t in base]
        got = dict(zip(["S"] + NAMES, [S[b:b + 1, h:h + 1]] + [a[b:b + 1, h:h + 1] for a in g]))
        check_outputs(got, scan_ref_fn(sl, gS[b:b + 1, h:h + 1], rule, ns), TOL_FP32,
                      prefix=f"({b},{h}):", widen=rule != 0)


def test_misaligned_tensors_take_the_exact_scan():
    """The tensor-core scan moves U, K, S, gS, dU and dK as 16-byte vectors
    (TMA boxes, float4); fp32 views that start 4 bytes into their storage are
    routed to the exact-fp32 kernels instead, with the same results."""
    pkg = load_pkg()
    base = pkg.workloads.scan_inputs(1, 2, 3, 128, C=64, seed=41)
    gS = torch.randn(base[0].shape, generator=torch.Generator().manual_seed(2))

    def shifted(t):   # same values, data pointer 4 bytes past a 16-byte boundary
        buf = torch.empty(t.numel() + 1, dtype=torch.float32, device="cuda")
        v = buf[1:].view(t.shape)
        v.copy_(t.float().cuda())
        assert v.data_ptr() % 16 == 4
        return v.requires_grad_(True)

    ins = [shifted(base[0]), shifted(base[1])] + [t.float().cuda().requires_grad_(True)
                                                  for t in base[2:]]

    def run():
        S = pkg.state_scan(*ins, 0, 3, pkg.GMDN_PREC_FAST)
        S.backward(gS.float().cuda())
        torch.cuda.synchronize()
        return S
    names = _launched(pkg, run)
    assert "scan_fwd_ieee" in names and "scan_fwd_tc" not in names, names
    for t in ins:
        t.grad = None
    S = run()
    S_ref, g_ref = run_kernel(pkg, base, gS, 0, 3, pkg.GMDN_PREC_FAST)
    assert (S.detach().cpu() - S_ref).abs().max().item() <= 1e-4 * S_ref.abs().max().item()
    for t, r in zip(ins, g_ref):
        assert (t.grad.cpu() - r).abs().max().item() <= 1e-4 * (r.abs().max().item() + 1e-30)
