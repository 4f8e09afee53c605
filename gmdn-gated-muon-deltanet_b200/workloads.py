"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (the reference publishes no dataset for this path).

Config 1-3 (B8 H16 T4096 dh128, chunk 64): q, k ~ N(0,1) then L2-normalised per
head vector; v ~ N(0,1); beta = sigmoid(N(0,1)); alpha = exp(-softplus(N(0,1)));
mu = sigmoid(N(0,1)); for adam mu = 0.9^(1/C), nu = 0.999^(1/C) per token so
the chunk products are 0.9 / 0.999; dO ~ N(0,1) from seed 1.  Everything is
drawn on the CPU from torch.Generator seeds, in that order.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

RULES = {"delta": 0, "muon": 1, "adam": 2}


@dataclass
class MixerInputs:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    alpha: torch.Tensor
    beta: torch.Tensor
    mu: torch.Tensor
    nu: torch.Tensor | None
    dO: torch.Tensor

    def to(self, device, act_dtype=torch.bfloat16):
        def mv(t, dt):
            return None if t is None else t.to(device=device, dtype=dt)
        return MixerInputs(mv(self.q, act_dtype), mv(self.k, act_dtype), mv(self.v, act_dtype),
                           mv(self.alpha, torch.float32), mv(self.beta, torch.float32),
                           mv(self.mu, torch.float32), mv(self.nu, torch.float32),
                           mv(self.dO, act_dtype))


def mixer_inputs(B: int, H: int, T: int, dh: int, rule: int, chunk: int = 64, seed: int = 0,
                 adam_fixed_moments: bool = True) -> MixerInputs:
    g = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(B, H, T, dh, generator=g), dim=-1)
    k = F.normalize(torch.randn(B, H, T, dh, generator=g), dim=-1)
    v = torch.randn(B, H, T, dh, generator=g)
    beta = torch.sigmoid(torch.randn(B, H, T, generator=g))
    alpha = torch.exp(-F.softplus(torch.randn(B, H, T, generator=g)))
    mu = torch.sigmoid(torch.randn(B, H, T, generator=g))
    nu = None
    if rule == 2:
        if adam_fixed_moments:
            mu = torch.full((B, H, T), 0.9 ** (1.0 / chunk))
            nu = torch.full((B, H, T), 0.999 ** (1.0 / chunk))
        else:
            nu = torch.sigmoid(torch.randn(B, H, T, generator=g))
    dO = torch.randn(B, H, T, dh, generator=torch.Generator().manual_seed(seed + 1))
    return MixerInputs(q, k, v, alpha, beta, mu, nu, dO)


def scan_inputs(B: int, H: int, N: int, dh: int, C: int = 64, seed: int = 0,
                family: str = "test"):
    """(U, K, a, b, m, n) on CPU, fp32.  family='test' follows the shape of the
    reference test fixture (test.py:28-38: normalised k, v/sqrt(dh), w in
    [0, 0.3), narrow gate ranges); 'wide' draws the gates from (0.01, 0.99)."""
    g = torch.Generator().manual_seed(seed)
    k = F.normalize(torch.randn(B, H, N, C, dh, generator=g), dim=-1)
    v = torch.randn(B, H, N, C, dh, generator=g) / dh ** 0.5
    w = torch.rand(B, H, N, C, generator=g) * 0.3
    K = (k * w.unsqueeze(-1)).mT @ k
    U = (v * w.unsqueeze(-1)).mT @ k
    if family == "test":
        ranges = ((0.2, 0.75), (0.5, 0.2), (0.5, 0.3), (0.2, 0.7))
        gates = [torch.rand(B, H, N, generator=g) * r + o for r, o in ranges]
    else:
        gates = [torch.rand(B, H, N, generator=g) * 0.98 + 0.01 for _ in range(4)]
    return [U, K] + gates
