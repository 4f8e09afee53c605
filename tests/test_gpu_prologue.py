"""GPU parity of the mixer prologue (conv + SiLU + q/k L2 norm + head layout,
gate sigmoids; train_ablation.py:124-140) against the CPU oracle, outputs and
every input gradient."""

import os

import pytest
import torch

import oracle
from conftest import load_pkg

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-300)).item()


def _check(pkg, u, w, b, gl, H, cot, tol, gtol):
    ug, wg, bg, glg = (t.cuda().requires_grad_(True) for t in (u, w, b, gl))
    outs = pkg.mixer_prologue(ug, wg, bg, glg, H)
    sum((o.float() * c.cuda().float()).sum() for o, c in zip(outs, cot)).backward()
    torch.cuda.synchronize()
    uc, wc, bc, glc = (t.clone().float().requires_grad_(True) for t in (u, w, b, gl))
    refs = oracle.mixer_prologue(uc, wc, bc, glc, H)
    sum((r * c.float()).sum() for r, c in zip(refs, cot)).backward()
    for name, o, r in zip(("q", "k", "v", "g"), outs, refs):
        assert o.dtype == u.dtype and o.shape == r.shape, name
        assert _rel(o, r) <= tol, f"{name} {_rel(o, r):.3e}"
    for name, gg, rg in (("du", ug.grad, uc.grad), ("dconv_w", wg.grad, wc.grad),
                         ("dconv_b", bg.grad, bc.grad), ("dgl", glg.grad, glc.grad)):
        assert _rel(gg, rg) <= gtol, f"{name} {_rel(gg, rg):.3e}"


@pytest.mark.parametrize("B,T,H,dh,nG,dt", [
    # wide strips (16-byte lanes, several heads a warp) where H allows, else one head a warp
    (2, 150, 2, 128, 3, torch.float32),    # T not a multiple of the 64-step strips
    (1, 64, 3, 64, 4, torch.float32),      # H 3: one head a warp
    (2, 96, 2, 32, 3, torch.float32),      # H 2 < 4 heads a warp: one head a warp
    (2, 256, 4, 128, 4, torch.bfloat16),
    (1, 130, 4, 64, 4, torch.bfloat16),    # four heads a warp, ragged last strip
    (2, 70, 8, 32, 3, torch.bfloat16),     # eight heads a warp
    (1, 67, 2, 64, 4, torch.float32),      # two heads a warp, fp32
    (1, 200, 4, 32, 3, torch.float32),
    (1, 128, 3, 128, 4, torch.bfloat16),   # H 3 at bf16 dh 128: one head a warp
])
def test_mixer_prologue_matches_oracle(B, T, H, dh, nG, dt):
    pkg = load_pkg()
    g = torch.Generator().manual_seed(B * 1000 + T + H * 10 + dh)
    D3 = 3 * H * dh
    u = torch.randn(B, T, D3, generator=g).to(dt)
    w = torch.randn(D3, 1, 4, generator=g) * 0.5
    b = torch.randn(D3, generator=g) * 0.1
    gl = torch.randn(B, T, nG * H, generator=g).to(dt)
    cot = [torch.randn(B, H, T, dh, generator=g).to(dt) for _ in range(3)]
    cot.append(torch.randn(nG, B, H, T, generator=g).to(dt))
    tol, gtol = (2e-5, 1e-4) if dt == torch.float32 else (2e-2, 3e-2)
    _check(pkg, u, w, b, gl, H, cot, tol, gtol)


def test_mixer_prologue_reference_fixtures():
    """The reference module's own forward (fp32 cases)."""
    pkg = load_pkg()
    cases = torch.load(os.path.join(GOLD, "prologue.pt"), weights_only=False)["cases"]
    for c in cases:
        if c["u"].dtype != torch.float32:
            continue
        ug, wg, bg, glg = (c[n].cuda().requires_grad_(True) for n in ("u", "conv_w", "conv_b", "gl"))
        q, k, v, g = pkg.mixer_prologue(ug, wg, bg, glg, c["n_heads"])
        for name, o in (("q", q), ("k", k), ("v", v), ("g", g)):
            assert _rel(o, c[name]) <= 2e-5, (c["name"], name)
        (sum((o * c["d" + n].cuda()).sum() for n, o in (("q", q), ("k", k), ("v", v), ("g", g)))
         ).backward()
        for name, gg in (("du", ug.grad), ("dgl", glg.grad), ("dconv_w", wg.grad),
                         ("dconv_b", bg.grad)):
            assert _rel(gg, c[name]) <= 1e-4, (c["name"], name)
