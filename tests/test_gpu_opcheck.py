"""torch.library registration of every op, and a compiled call.

The trainer compiles its model (``--compile``: torch.compile(dynamic=False),
train_ablation.py:420-422, 577), so every op must have a correct schema, fake
(meta) kernel and autograd registration.  torch.library.opcheck checks them
against the real kernels; the dynamic-shape check is left out because the
fake kernels size their scratch through the C ABI with concrete ints, as the
trainer's static compile does.
"""
import pytest
import torch

from conftest import load_pkg

pytestmark = pytest.mark.gpu

UTILS = ("test_schema", "test_autograd_registration", "test_faketensor",
         "test_aot_dispatch_static")


def _gates(B, H, T, n, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.sigmoid(torch.randn(B, H, T, generator=g)).cuda() for _ in range(n)]


@pytest.mark.parametrize("rule,dh,prec", [(0, 128, 1), (1, 128, 1), (2, 64, 1), (0, 32, 0)])
def test_opcheck_chunk_ops(rule, dh, prec):
    pkg = load_pkg()
    B, H, T = 1, 2, 128
    g = torch.Generator().manual_seed(3)
    dt = torch.bfloat16 if prec == 1 else torch.float32
    q, k, v = (torch.nn.functional.normalize(torch.randn(B, H, T, dh, generator=g), dim=-1)
               .to("cuda", dt).requires_grad_(True) for _ in range(3))
    alpha, beta, mu, nu = (t.requires_grad_(True) for t in _gates(B, H, T, 4, 4))
    nu = nu if rule == 2 else None
    args = (q, k, v, alpha, beta, mu, nu, rule, 3, 64, prec)
    torch.library.opcheck(torch.ops.gmdn.chunk_fwd.default, args, test_utils=UTILS)
    o, saved = torch.ops.gmdn.chunk_fwd(*args)
    dO = torch.randn(B, H, T, dh, generator=g).to("cuda", dt)
    bargs = (q.detach(), k.detach(), v.detach(), alpha.detach(), beta.detach(), mu.detach(),
             None if nu is None else nu.detach(), dO, saved, rule, 3, 64, prec)
    torch.library.opcheck(torch.ops.gmdn.chunk_bwd.default, bargs,
                          test_utils=("test_schema", "test_faketensor"))


@pytest.mark.parametrize("rule,prec", [(0, 1), (2, 0), (1, 0)])
def test_opcheck_scan_ops(rule, prec):
    pkg = load_pkg()
    base = [t.cuda().requires_grad_(True) for t in pkg.workloads.scan_inputs(1, 2, 3, 128, seed=6)]
    args = (*base, rule, 3, prec)
    torch.library.opcheck(torch.ops.gmdn.state_scan_fwd.default, args, test_utils=UTILS)


def test_opcheck_epilogue_and_prologue_ops():
    pkg = load_pkg()
    g = torch.Generator().manual_seed(8)
    o = torch.randn(1, 2, 64, 64, generator=g).to("cuda", torch.bfloat16).requires_grad_(True)
    w = (1 + 0.1 * torch.randn(64, generator=g)).cuda().requires_grad_(True)
    torch.library.opcheck(torch.ops.gmdn.head_rmsnorm_fwd.default, (o, w, -1.0, True),
                          test_utils=UTILS)
    D, H = 128, 2
    u = torch.randn(1, 64, 3 * D, generator=g).to("cuda", torch.bfloat16).requires_grad_(True)
    cw = (0.5 * torch.randn(3 * D, 1, 4, generator=g)).cuda().requires_grad_(True)
    cb = (0.1 * torch.randn(3 * D, generator=g)).cuda().requires_grad_(True)
    gl = torch.randn(1, 64, 3 * H, generator=g).to("cuda", torch.bfloat16).requires_grad_(True)
    torch.library.opcheck(torch.ops.gmdn.mixer_prologue_fwd.default, (u, cw, cb, gl, H),
                          test_utils=UTILS)


@pytest.mark.parametrize("rule", [0, 1])
def test_compiled_mixer_core_matches_eager(rule):
    """One torch.compile'd (default mode, static shapes) forward + backward of
    the mixer core on the tensor-core path matches the eager call: the compiled
    graph calls the same ops on the same inputs."""
    pkg = load_pkg()
    torch._dynamo.reset()
    inp = pkg.workloads.mixer_inputs(1, 2, 256, 128, rule=rule, seed=31)
    names = ["q", "k", "v", "alpha", "beta", "mu"]

    def leaves():
        return [getattr(inp, n).to("cuda", torch.bfloat16 if n in "qkv" else torch.float32)
                .requires_grad_(True) for n in names]

    def fn(q, k, v, alpha, beta, mu):
        o = pkg.chunk_fast_weight(q, k, v, alpha, beta, mu, None, rule, 3, 64,
                                  pkg.GMDN_PREC_FAST)
        return (o.float() * o.float()).sum()

    dO_seed = leaves()
    eager = fn(*dO_seed)
    eager.backward()
    compiled = torch.compile(fn, dynamic=False)
    cl = leaves()
    out = compiled(*cl)
    out.backward()
    torch.cuda.synchronize()
    # the compiled graph sums the loss in its own order (a relative 1e-7), so
    # the cotangent dO = 2 o it feeds the op differs in the last bits
    assert torch.allclose(out, eager, rtol=1e-5)
    for a, b in zip(cl, dO_seed):
        ref = b.grad.float().abs().max().item()
        if ref == 0.0:       # a gate the rule never reads: zeros both ways
            assert a.grad.abs().max().item() == 0.0
            continue
        e = (a.grad.float() - b.grad.float()).abs().max().item() / ref
        assert e < 1e-3, e
