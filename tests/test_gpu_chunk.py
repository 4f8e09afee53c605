"""GPU parity of the mixer core (phases 1-3, train_ablation.py:142-187)
against the CPU oracle, forward output and every input gradient."""
import os

import pytest
import torch

from conftest import load_pkg
from oracle_runs import mixer_oracle
from parity import TOL_BF16, TOL_FP32, check_outputs, perturb

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
GRADS = ["dq", "dk", "dv", "dalpha", "dbeta", "dmu", "dnu"]


def run_kernel(pkg, inp, rule, ns, chunk, precision, act_dtype):
    names = ["q", "k", "v", "alpha", "beta", "mu", "nu"]
    ins = []
    for n in names:
        t = getattr(inp, n)
        if t is not None:
            dt = act_dtype if n in ("q", "k", "v") else torch.float32
            t = t.detach().to("cuda", dt).requires_grad_(True)
        ins.append(t)
    o = pkg.chunk_fast_weight(*ins, rule, ns, chunk, precision)
    o.backward(inp.dO.to("cuda", act_dtype))
    torch.cuda.synchronize()
    grads = {"d" + n: t.grad.detach().float().cpu() for n, t in zip(names, ins) if t is not None}
    return o.detach().float().cpu(), grads


def round_inputs(inp, act_dtype):
    """Inputs as the kernel sees them (activations rounded to act_dtype)."""
    import copy
    r = copy.copy(inp)
    for n in ("q", "k", "v", "dO"):
        setattr(r, n, getattr(inp, n).to(act_dtype).float())
    return r


def mixer_ref_fn(ri, rule, ns, chunk, gold=None):
    """ref_fn for parity.check_outputs over the (rounded) inputs `ri`."""
    import copy

    def fn(dtype, seed):
        if dtype == torch.float64 and gold is not None:
            return gold
        x = ri
        if seed is not None:
            x = copy.copy(ri)
            for i, n in enumerate(("q", "k", "v", "alpha", "beta", "mu", "nu")):
                setattr(x, n, perturb(getattr(ri, n), seed * 10 + i))
        o, g = mixer_oracle(x, rule, ns, chunk, dtype)
        return {"o": o, **g}
    return fn


def compare(pkg, inp, rule, ns, chunk, precision, act_dtype, tol, sl=None):
    o, g = run_kernel(pkg, inp, rule, ns, chunk, precision, act_dtype)
    ri = round_inputs(inp, act_dtype)
    if sl is not None:
        ri = slice_inputs(ri, *sl)
        o = o[sl[0]:sl[0] + 1, sl[1]:sl[1] + 1]
        g = {k: v[sl[0]:sl[0] + 1, sl[1]:sl[1] + 1] for k, v in g.items()}
    check_outputs({"o": o, **g}, mixer_ref_fn(ri, rule, ns, chunk), tol,
                  widen=(tol == TOL_FP32 and rule != 0))


def slice_inputs(inp, b, h):
    import copy
    r = copy.copy(inp)
    for n in ("q", "k", "v", "alpha", "beta", "mu", "nu", "dO"):
        t = getattr(inp, n)
        if t is not None:
            setattr(r, n, t[b:b + 1, h:h + 1])
    return r


CONFIG0 = dict(B=2, H=4, T=256, dh=64)


@pytest.mark.parametrize("rule,ns", [(0, 3), (1, 3), (1, 5), (2, 3)])
@pytest.mark.parametrize("chunk", [32, 64])
def test_config0_fp32_ieee(rule, ns, chunk):
    """Config 0 shape (B2 H4 T256 dh64) in fp32: the 1e-4 bar."""
    pkg = load_pkg()
    inp = pkg.workloads.mixer_inputs(**CONFIG0, rule=rule, chunk=chunk, seed=rule)
    compare(pkg, inp, rule, ns, chunk, pkg.GMDN_PREC_IEEE, torch.float32, TOL_FP32)


@pytest.mark.parametrize("rule,ns", [(0, 3), (1, 5), (2, 3)])
@pytest.mark.parametrize("precision", [0, 1])
def test_bf16_inputs(rule, ns, precision):
    """bf16 activations (the autocast trainer): the 2e-2 bar."""
    pkg = load_pkg()
    inp = pkg.workloads.mixer_inputs(2, 4, 512, 128, rule=rule, seed=20 + rule)
    compare(pkg, inp, rule, ns, 64, precision, torch.bfloat16, TOL_BF16)


@pytest.mark.parametrize("dh", [16, 32])
def test_small_head_dims(dh):
    pkg = load_pkg()
    for rule, ns in ((0, 3), (1, 3), (2, 3)):
        inp = pkg.workloads.mixer_inputs(1, 3, 128, dh, rule=rule, seed=40 + dh + rule)
        compare(pkg, inp, rule, ns, 64, pkg.GMDN_PREC_IEEE, torch.float32, TOL_FP32)


def test_trainer_gate_regime():
    """alpha close to 1 (the trainer's gate prior, train_ablation.py:105) so the
    decay term a_c is exercised, sigmoid nu for adam."""
    pkg = load_pkg()
    for rule, ns in ((0, 3), (1, 3), (2, 3)):
        inp = pkg.workloads.mixer_inputs(1, 2, 256, 64, rule=rule, seed=50 + rule,
                                         adam_fixed_moments=False)
        inp.alpha = 0.9 + 0.1 * inp.alpha
        compare(pkg, inp, rule, ns, 64, pkg.GMDN_PREC_IEEE, torch.float32, TOL_FP32)


def test_golden_fixtures():
    """The reference's own FastWeightMixer phases 1-3 (tests/golden/mixer.pt)."""
    pkg = load_pkg()
    import copy
    for case in torch.load(os.path.join(GOLD, "mixer.pt"))["cases"]:
        inp = pkg.workloads.MixerInputs(case["q"], case["k"], case["v"], case["alpha"],
                                        case["beta"], case["mu"], case["nu"], case["dO"])
        o, g = run_kernel(pkg, inp, case["rule"], case["ns"], case["chunk"],
                          pkg.GMDN_PREC_IEEE, torch.float32)
        ri = round_inputs(copy.copy(inp), torch.float32)
        gold = {"o": case["o"], **{n: case[n] for n in GRADS if case.get(n) is not None}}
        check_outputs({"o": o, **g}, mixer_ref_fn(ri, case["rule"], case["ns"], case["chunk"], gold),
                      TOL_FP32, prefix=case["name"] + ":", widen=case["rule"] != 0)


@pytest.mark.parametrize("rule,ns", [(0, 3), (2, 3), (1, 5)])
def test_config1_full_size_slices(rule, ns):
    """B8 H16 T4096 dh128 bf16 (configs 1-3): slices of the full run against the
    oracle on the same slice."""
    pkg = load_pkg()
    inp = pkg.workloads.mixer_inputs(8, 16, 4096, 128, rule=rule, seed=0)
    for sl in ((0, 0), (7, 15)):
        compare(pkg, inp, rule, ns, 64, pkg.GMDN_PREC_FAST, torch.bfloat16, TOL_BF16, sl=sl)


@pytest.mark.parametrize("B,H,T,rule,ns", [
    (1, 1, 64, 0, 3), (1, 1, 64, 1, 5), (1, 1, 64, 2, 3),   # one chunk-tile (N = 1)
    (1, 1, 128, 1, 5),                                       # two tiles
    (1, 1, 149 * 64, 0, 3),                                  # 149 tiles: one CTA walks two
    (1, 3, 99 * 64, 2, 3),                                   # 297 tiles: one CTA walks three
])
def test_tile_scheduling_edges(B, H, T, rule, ns):
    """Tile counts around the persistent token-gradient kernel's grid (one CTA
    per SM, 148 on B200): fewer tiles than CTAs, and CTAs walking one, two or
    three tiles, which exercises the q/k load-ahead buffers, the S_j / Gb_j
    tile swap, the per-parity TMEM release and the deferred gate gradients of
    the last tile."""
    pkg = load_pkg()
    inp = pkg.workloads.mixer_inputs(B, H, T, 128, rule=rule, seed=60 + rule)
    compare(pkg, inp, rule, ns, 64, pkg.GMDN_PREC_FAST, torch.bfloat16, TOL_BF16)


def test_precisions_agree_closely():
    pkg = load_pkg()
    inp = pkg.workloads.mixer_inputs(2, 2, 256, 128, rule=0, seed=77)
    o0, g0 = run_kernel(pkg, inp, 0, 3, 64, 0, torch.bfloat16)
    o1, g1 = run_kernel(pkg, inp, 0, 3, 64, 1, torch.bfloat16)
    from parity import rel
    assert rel(o1, o0) < 2e-2
    for k in g0:
        assert rel(g1[k], g0[k]) < 2e-2, k


@pytest.mark.parametrize("rule,ns", [(0, 3), (2, 3), (1, 5)])
def test_full_size_runs_are_repeatable(rule, ns):
    """Repeated fwd+bwd at config-1 size must give bitwise-identical o, dq, dk,
    dv: every product and reduction is in a fixed order, so a difference means
    a hand-off race (a product issued before its operands landed).  Gate
    cotangents are summed with float atomics across CTAs and only have to
    agree closely."""
    pkg = load_pkg()
    inp = pkg.workloads.mixer_inputs(8, 16, 4096, 128, rule=rule, seed=3)
    o0, g0 = run_kernel(pkg, inp, rule, ns, 64, pkg.GMDN_PREC_FAST, torch.bfloat16)
    for rep in range(5):
        o, g = run_kernel(pkg, inp, rule, ns, 64, pkg.GMDN_PREC_FAST, torch.bfloat16)
        assert torch.equal(o, o0), f"run {rep + 1}: o differs"
        for n in ("dq", "dk", "dv"):
            assert torch.equal(g[n], g0[n]), f"run {rep + 1}: {n} differs"
        for n in ("dalpha", "dbeta", "dmu", "dnu"):
            if n in g0:
                scale = g0[n].abs().max().item() + 1e-30
                assert (g[n] - g0[n]).abs().max().item() <= 1e-5 * scale, f"run {rep + 1}: {n}"


def _launched(pkg, fn):
    """Names of the library kernels `fn` launches (the library's own per-launch
    records)."""
    L = pkg._lib
    L.prof_report()
    L.prof_enable(True)
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        L.prof_enable(False)
    return set(L.prof_report())


@pytest.mark.parametrize("rule,ns", [(0, 3), (1, 3), (1, 5), (2, 3)])
def test_dh64_tensor_core_slices(rule, ns):
    """dh 64, the trainer's default head (d_model 768 / 12 heads,
    train_ablation.py:551-553; test.py:100), on the tensor-core kernels at the
    config-4 per-layer scan shape B8 H12 T2048 bf16: slices of the full run
    against the oracle on the same slice, and the kernels that ran are the
    tcgen05 ones."""
    pkg = load_pkg()
    inp = pkg.workloads.mixer_inputs(8, 12, 2048, 64, rule=rule, seed=90 + rule)
    names = _launched(pkg, lambda: run_kernel(pkg, inp, rule, ns, 64, pkg.GMDN_PREC_FAST,
                                              torch.bfloat16))
    fwd = "chunk_fwd_muon_tc" if rule == 1 else "chunk_fwd_tc"
    if rule == 0:   # 96 sequences < 148 SMs: the fused chain + token-gradient backward
        assert {fwd, "chunk_bwd_fused_tc"} <= names, names
    else:
        bw1 = "chunk_bwd1_muon_tc" if rule == 1 else "chunk_bwd1_tc"
        assert {fwd, bw1, "chunk_bwd2_tc"} <= names, names
    for sl in ((0, 0), (7, 11)):
        compare(pkg, inp, rule, ns, 64, pkg.GMDN_PREC_FAST, torch.bfloat16, TOL_BF16, sl=sl)


@pytest.mark.parametrize("rule,ns", [(0, 3), (1, 5), (2, 3)])
def test_dh64_tensor_core_whole_batch(rule, ns):
    """dh 64 on the tensor cores, every (b, h) of a small batch against the
    oracle (N = 1, 2 and 5 chunks)."""
    pkg = load_pkg()
    for T in (64, 128, 320):
        inp = pkg.workloads.mixer_inputs(2, 3, T, 64, rule=rule, seed=95 + rule + T)
        compare(pkg, inp, rule, ns, 64, pkg.GMDN_PREC_FAST, torch.bfloat16, TOL_BF16)


def test_config3_long_slice():
    """Config 3-long (B1 H16 T65536 = 1024 chunks, adam
    configs[3]) on the tensor-core path: one head of the full run against the
    oracle on that head, at the flat bf16 bar."""
    pkg = load_pkg()
    inp = pkg.workloads.mixer_inputs(1, 16, 65536, 128, rule=2, seed=0)
    compare(pkg, inp, 2, 3, 64, pkg.GMDN_PREC_FAST, torch.bfloat16, TOL_BF16, sl=(0, 7))
