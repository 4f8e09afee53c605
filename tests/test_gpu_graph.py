"""CUDA-graph capture of the ops: a fwd+bwd of the mixer core, of the scan
and of the prologue/epilogue captured once and replayed gives the results of
plain calls (the library enqueues everything on the caller's stream, with no
host synchronisation and no allocation outside torch's allocator, so a
training loop can replay it without the host's per-launch work)."""
import pytest
import torch

from conftest import load_pkg

pytestmark = pytest.mark.gpu


def _capture(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    torch.cuda.synchronize()
    return g, out


def _close(a, b, exact):
    if exact:
        return torch.equal(a, b)
    scale = b.float().abs().max().item() + 1e-30
    return (a.float() - b.float()).abs().max().item() <= 1e-5 * scale


@pytest.mark.parametrize("rule", [0, 1, 2])
def test_mixer_core_graph_replay(rule):
    pkg = load_pkg()
    inp = pkg.workloads.mixer_inputs(1, 4, 512, 128, rule=rule, seed=60 + rule)
    names = ["q", "k", "v", "alpha", "beta", "mu"] + (["nu"] if rule == 2 else [])
    leaves = [getattr(inp, n).to("cuda", torch.bfloat16 if n in "qkv" else torch.float32)
              .requires_grad_(True) for n in names]
    dO = inp.dO.to("cuda", torch.bfloat16)

    def step():
        nu = leaves[6] if rule == 2 else None
        o = pkg.chunk_fast_weight(*leaves[:6], nu, rule, 3, 64, pkg.GMDN_PREC_FAST)
        return (o.detach(),) + torch.autograd.grad(o, leaves, dO)

    g, out = _capture(step)
    with torch.no_grad():
        for t in leaves:   # new input values: the replay must read them
            t.mul_(0.5 if t.dtype == torch.bfloat16 else 1.0)
    g.replay()
    ref = step()
    torch.cuda.synchronize()
    # o, dq, dk, dv bit for bit; gate gradients sum per-CTA partials with atomics
    for i, (a, b) in enumerate(zip(out, ref)):
        assert _close(a, b, exact=i < 4), (rule, i)


def test_scan_and_pieces_graph_replay():
    pkg = load_pkg()
    base = [t.cuda().requires_grad_(True) for t in pkg.workloads.scan_inputs(1, 2, 4, 128, seed=61)]
    gS = torch.randn(base[0].shape, generator=torch.Generator().manual_seed(1)).cuda()

    def scan_step():
        S = pkg.state_scan(*base, 0, 3, pkg.GMDN_PREC_FAST)
        return (S.detach(),) + torch.autograd.grad(S, base, gS)

    g, out = _capture(scan_step)
    g.replay()
    ref = scan_step()
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(out, ref)):
        assert _close(a, b, exact=i < 3), i

    gen = torch.Generator().manual_seed(62)
    o = torch.randn(1, 2, 256, 64, generator=gen).to("cuda", torch.bfloat16).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(64, generator=gen)).cuda().requires_grad_(True)
    dy = torch.randn(1, 256, 128, generator=gen).to("cuda", torch.bfloat16)

    def epi_step():
        y = pkg.head_rmsnorm(o, w)
        return (y.detach(),) + torch.autograd.grad(y, (o, w), dy)

    g, out = _capture(epi_step)
    g.replay()
    ref = epi_step()
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(out, ref)):
        assert _close(a, b, exact=i < 2), i
