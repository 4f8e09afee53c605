"""GPU parity of the mixer epilogue (per-head RMSNorm into the (B, T, D) layout,
train_ablation.py:188-189) against the CPU oracle, output and both gradients."""

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


def _tol(dt):
    # fp32: fp32 evaluations in another order; bf16: one bf16 rounding step
    return 2e-5 if dt == torch.float32 else 8e-3


def _run(pkg, o, w, dy, out_dtype):
    og = o.cuda().requires_grad_(True)
    wg = w.cuda().requires_grad_(True)
    y = pkg.head_rmsnorm(og, wg, None, out_dtype)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    return y.detach().cpu(), og.grad.cpu(), wg.grad.cpu()


def _oracle(o, w, dy, out_dtype):
    oc = o.clone().requires_grad_(True)
    wc = w.clone().requires_grad_(True)
    y = oracle.head_rmsnorm(oc, wc, None, out_dtype)
    (y.double() * dy.double()).sum().backward()
    return y.detach(), oc.grad, wc.grad


@pytest.mark.parametrize("B,H,T,dh,in_dt,out_dt", [
    (2, 3, 50, 128, torch.float32, torch.float32),
    (2, 3, 50, 128, torch.bfloat16, torch.bfloat16),
    (2, 3, 50, 128, torch.bfloat16, torch.float32),
    (1, 2, 33, 64, torch.float32, torch.float32),
    (1, 2, 17, 32, torch.bfloat16, torch.bfloat16),
    (1, 4, 4096, 128, torch.bfloat16, torch.bfloat16),   # many blocks, grid-stride rows
    # wide rows (several rows a warp step): runs crossing (b, h), odd row counts, T < rows a step
    (3, 5, 1, 32, torch.bfloat16, torch.bfloat16),        # T 1: every step crosses heads
    (2, 3, 7, 64, torch.bfloat16, torch.bfloat16),
    (1, 3, 3001, 64, torch.float32, torch.bfloat16),
    (2, 2, 999, 128, torch.bfloat16, torch.float32),
    (8, 16, 512, 128, torch.bfloat16, torch.bfloat16),    # 65,536 rows over the whole grid
])
def test_head_rmsnorm_matches_oracle(B, H, T, dh, in_dt, out_dt):
    pkg = load_pkg()
    g = torch.Generator().manual_seed(B * 1000 + H * 100 + T + dh)
    scale = torch.exp(torch.randn(B, H, T, 1, generator=g))
    o = (torch.randn(B, H, T, dh, generator=g) * scale).to(in_dt)
    w = 1.0 + 0.5 * torch.randn(dh, generator=g)
    dy = torch.randn(B, T, H * dh, generator=g).to(out_dt)
    y, d_o, dw = _run(pkg, o, w, dy, out_dt)
    ry, rdo, rdw = _oracle(o, w, dy, out_dt)
    assert y.dtype == ry.dtype and y.shape == ry.shape
    assert d_o.dtype == in_dt and dw.dtype == torch.float32
    tol = _tol(in_dt)
    # y is rounded to the output dtype last: a bf16 output is held to the bf16 bound
    assert _rel(y, ry) <= max(tol, _tol(out_dt)), f"y {_rel(y, ry):.3e}"
    assert _rel(d_o, rdo) <= tol, f"d_o {_rel(d_o, rdo):.3e}"
    assert _rel(dw, rdw) <= max(tol, 1e-4), f"dweight {_rel(dw, rdw):.3e}"


def test_head_rmsnorm_reference_fixtures():
    """The reference module's own nn.RMSNorm outputs (fp32 and bf16 cases)."""
    pkg = load_pkg()
    cases = torch.load(os.path.join(GOLD, "epilogue.pt"), weights_only=False)["cases"]
    for c in cases:
        if c["o"].dtype == torch.float64:
            continue
        y, d_o, dw = _run(pkg, c["o"], c["weight"].float(), c["dy"], c["out_dtype"])
        tol = _tol(c["o"].dtype)
        assert _rel(y, c["y"]) <= tol, c["name"]
        assert _rel(d_o, c["d_o"]) <= tol, c["name"]
        assert _rel(dw, c["dweight"]) <= max(tol, 1e-4), c["name"]


def test_head_rmsnorm_rejects_bad_shapes():
    pkg = load_pkg()
    o = torch.zeros(1, 2, 8, 48, device="cuda")
    with pytest.raises(ValueError):
        pkg.head_rmsnorm(o, torch.ones(48, device="cuda"))
    lib = pkg._lib.lib
    import ctypes
    rc = lib.gmdn_head_rmsnorm_fwd(ctypes.c_void_p(o.data_ptr()), ctypes.c_void_p(o.data_ptr()),
                                   ctypes.c_void_p(o.data_ptr()), 1, 2, 8, 48, -1.0, 1, 1,
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 2   # GMDN_ERR_UNSUPPORTED
