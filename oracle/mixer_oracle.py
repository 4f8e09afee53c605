"""CPU restatement of the reference's mixer core, phases 1-3 (TEST ORACLE).

Reference: ``train_ablation.py`` of cloud-777-boy/GMDN-GATED-MUON-DELTANET,
``FastWeightMixer.forward`` lines 142-187:

  * per-rule token weights w                     -- train_ablation.py:150-158
  * A = tril(q k^T) * beta_col, Kw, Uv, Qt, Ov   -- train_ablation.py:160-167
  * chunk gate scalars a_c, b_c, mu_c, nu_c      -- train_ablation.py:169-175
  * phase 2 state scan                           -- train_ablation.py:179-182
  * o = Qt S^T + Ov                              -- train_ablation.py:184-187

The projections / conv / gate sigmoid before line 142 and the RMSNorm / output
projection after line 187 are not part of the scanned path and are not
restated.  Everything is computed in the dtype of the inputs (fp32 for the
parity bar, fp64 as ground truth); backward is torch autograd of this forward.
"""

from __future__ import annotations

import torch

from .scan_oracle import scan_forward

RULES = {"delta": 0, "muon": 1, "adam": 2}


def _log_clamped(x: torch.Tensor) -> torch.Tensor:
    return torch.log(x.clamp_min(1e-6))


def token_weights(beta_c: torch.Tensor, mu_c: torch.Tensor, rule: int) -> torch.Tensor:
    """w inside the chunk gradient, (B, H, N, C) (train_ablation.py:151-158).

    delta: w_s = beta_s.  muon: w_s = prod_{t>s} mu_t (log-space suffix sum of
    clamped mu, minus the own term).  adam: w_s = 1.
    """
    if rule == 0:
        return beta_c
    if rule == 1:
        lm = _log_clamped(mu_c)
        suffix = torch.flip(torch.cumsum(torch.flip(lm, [-1]), -1), [-1])
        return torch.exp(suffix - lm)
    return torch.ones_like(beta_c)


def chunk_gate_scalars(alpha_c, beta_c, mu_c, nu_c):
    """(a_c, b_c, mu_c, nu_c) per chunk, each (B, H, N) (train_ablation.py:170-175).
    nu_c is all ones when the rule has no nu gate (train_ablation.py:180)."""
    a = torch.exp(_log_clamped(alpha_c).sum(-1))
    b = beta_c.mean(-1)
    m = torch.exp(_log_clamped(mu_c).sum(-1))
    if nu_c is None:
        n = torch.ones_like(a)
    else:
        n = torch.exp(_log_clamped(nu_c).sum(-1))
    return a, b, m, n


def mixer_core_forward(q, k, v, alpha, beta, mu, nu, rule: int, ns: int,
                       chunk: int = 64, return_states: bool = False):
    """o (B, H, T, dh) from q, k, v (B, H, T, dh) and gates (B, H, T).

    ``nu`` is used only by rule 2 (adam) and may be None otherwise.
    """
    Bsz, H, T, dh = q.shape
    C = chunk
    if T % C:
        raise ValueError("T must be a multiple of the chunk size")
    N = T // C
    qn = q.reshape(Bsz, H, N, C, dh)
    kn = k.reshape(Bsz, H, N, C, dh)
    vn = v.reshape(Bsz, H, N, C, dh)
    an = alpha.reshape(Bsz, H, N, C)
    bn = beta.reshape(Bsz, H, N, C)
    mn = mu.reshape(Bsz, H, N, C)
    nun = nu.reshape(Bsz, H, N, C) if (rule == 2 and nu is not None) else None

    w = token_weights(bn, mn, rule)
    causal = torch.ones(C, C, dtype=torch.bool, device=q.device).tril()
    A = ((qn @ kn.transpose(-1, -2)) * bn.unsqueeze(-2)).masked_fill(~causal, 0.0)
    Kw = (kn * w.unsqueeze(-1)).transpose(-1, -2) @ kn
    Uv = (vn * w.unsqueeze(-1)).transpose(-1, -2) @ kn
    Qt = qn - A @ kn
    Ov = A @ vn

    a_c, b_c, m_c, n_c = chunk_gate_scalars(an, bn, mn, nun)
    states = scan_forward(Uv, Kw, a_c, b_c, m_c, n_c, rule, ns)
    o = (Qt @ states.transpose(-1, -2) + Ov).reshape(Bsz, H, T, dh)
    if return_states:
        return o, states
    return o
