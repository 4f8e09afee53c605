"""CPU oracle of the mixer epilogue (TEST INFRASTRUCTURE ONLY).

train_ablation.py:188-189 applies ``self.norm(o).to(x.dtype)`` with
``self.norm = nn.RMSNorm(dh)`` (train_ablation.py:97) and then views the result
as (B, T, D) for the output projection.  nn.RMSNorm is torch's (2.11 here);
its rms_norm, restated: the input is upcast to the computation dtype (fp32 for
bf16 / fp32 input, fp64 for fp64), eps defaults to that dtype's machine
epsilon, y = x * rsqrt(mean(x^2, -1) + eps) * weight, cast back to the input
dtype.  The fixtures of tests/golden/epilogue.pt come from the reference
module's own ``norm`` and pin this restatement.
"""

from __future__ import annotations

import torch


def head_rmsnorm(o: torch.Tensor, weight: torch.Tensor, eps: float | None = None,
                 out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """o (B, H, T, dh) -> (B, T, H * dh): rms_norm over dh, then the reference's
    dtype conversion and head transpose.  Differentiable (autograd gives the
    reference's backward)."""
    B, H, T, dh = o.shape
    comp = torch.float64 if o.dtype == torch.float64 else torch.float32
    if eps is None:
        eps = torch.finfo(comp).eps
    x = o.to(comp)
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight.to(comp)
    y = y.to(o.dtype).to(out_dtype or o.dtype)
    return y.transpose(1, 2).reshape(B, T, H * dh)
