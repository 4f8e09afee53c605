"""GPU test of ``patch_mixer``'s forward: a module with FastWeightMixer's
attribute layout (train_ablation.py:84-100) runs integration.mixer_forward on
CUDA (phases 1-3 on the chunk op, the per-head RMSNorm on the epilogue op) and
is compared with the same lines evaluated on the CPU with the oracle mixer
core and the module's own torch norm."""

import importlib

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import oracle
from conftest import PKG_NAME, load_pkg

pytestmark = pytest.mark.gpu


class _MixerLayout(nn.Module):
    """The attributes integration.mixer_forward reads (train_ablation.py:84-100)."""

    def __init__(self, D, H, inner, chunk, ns):
        super().__init__()
        self.h, self.dh = H, D // H
        self.inner, self.chunk, self.ns_steps = inner, chunk, ns
        self.qkv = nn.Linear(D, 3 * D, bias=False)
        self.conv = nn.Conv1d(3 * D, 3 * D, 4, groups=3 * D, padding=3)
        self.n_gates = 4 if inner == "adam" else 3
        self.gates = nn.Linear(D, self.n_gates * H, bias=True)
        self.norm = nn.RMSNorm(self.dh)
        self.out = nn.Linear(D, D, bias=False)
        with torch.no_grad():
            self.norm.weight.copy_(1.0 + 0.3 * torch.randn(self.dh))


def _cpu_forward(m, x):
    B, T, D = x.shape
    H, dh = m.h, m.dh
    qkv = m.conv(m.qkv(x).transpose(1, 2))[..., :T].transpose(1, 2)
    q, k, v = F.silu(qkv).chunk(3, dim=-1)
    q = F.normalize(q.reshape(B, T, H, dh).transpose(1, 2), dim=-1)
    k = F.normalize(k.reshape(B, T, H, dh).transpose(1, 2), dim=-1)
    v = v.reshape(B, T, H, dh).transpose(1, 2)
    g = torch.sigmoid(m.gates(x)).view(B, T, m.n_gates, H).permute(2, 0, 3, 1)
    nu = g[3] if m.n_gates == 4 else None
    rule = {"delta": 0, "muon": 1, "adam": 2}[m.inner]
    o = oracle.mixer_core_forward(q, k, v, g[0], g[1], g[2], nu, rule, m.ns_steps, m.chunk)
    o = m.norm(o).to(x.dtype)
    return m.out(o.transpose(1, 2).reshape(B, T, D))


@pytest.mark.parametrize("inner", ["delta", "adam"])
def test_patched_mixer_forward_matches_cpu(inner):
    load_pkg()
    integ = importlib.import_module(PKG_NAME + ".integration")
    torch.manual_seed(11)
    m = _MixerLayout(256, 2, inner, 64, 3)
    x = torch.randn(1, 128, 256) * 0.5
    xc = x.clone().requires_grad_(True)
    ref = _cpu_forward(m, xc)
    ref.backward(torch.ones_like(ref))
    mg = m.cuda()
    xg = x.cuda().requires_grad_(True)
    y = integ.mixer_forward(mg, xg)
    y.backward(torch.ones_like(y))
    torch.cuda.synchronize()
    err = (y.detach().cpu() - ref.detach()).abs().max() / ref.abs().max()
    assert err < 2e-3, f"y rel err {err:.3e}"
    gerr = (xg.grad.cpu() - xc.grad).abs().max() / xc.grad.abs().max()
    assert gerr < 5e-3, f"dx rel err {gerr:.3e}"
    wg = mg.norm.weight.grad.cpu()
    assert torch.isfinite(wg).all() and wg.abs().max() > 0
