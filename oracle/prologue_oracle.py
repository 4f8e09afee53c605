"""CPU oracle of the mixer prologue (TEST INFRASTRUCTURE ONLY).

train_ablation.py:124-140 after the two projections u = self.qkv(x) and
gl = self.gates(x), restated: a depthwise Conv1d of kernel 4 with padding 3
truncated to the first T outputs (causal), SiLU, the split into q, k, v by
head, F.normalize of q and k over dh (eps 1e-12), and sigmoid gates laid out
(nG, B, H, T).  The fixtures of tests/golden/prologue.pt, recorded from the
reference module's own forward, pin this restatement.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def mixer_prologue(u: torch.Tensor, conv_w: torch.Tensor, conv_b: torch.Tensor,
                   gl: torch.Tensor, n_heads: int):
    """q, k, v (B, H, T, dh) and g (nG, B, H, T); differentiable."""
    B, T, D3 = u.shape
    H, dh = n_heads, D3 // 3 // n_heads
    z = F.conv1d(u.transpose(1, 2), conv_w, conv_b, padding=3, groups=D3)[..., :T]
    s = F.silu(z.transpose(1, 2))
    q, k, v = s.chunk(3, dim=-1)
    q = F.normalize(q.reshape(B, T, H, dh).transpose(1, 2), dim=-1)
    k = F.normalize(k.reshape(B, T, H, dh).transpose(1, 2), dim=-1)
    v = v.reshape(B, T, H, dh).transpose(1, 2)
    g = torch.sigmoid(gl).view(B, T, gl.shape[-1] // H, H).permute(2, 0, 3, 1)
    return q, k, v, g
