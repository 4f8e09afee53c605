"""Emulation of the reference's own GPU numerics on the CPU (TEST ORACLE).

The parity bar for bf16 runs has two parts: within 2e-2 of the naive fp32
recurrence, and no worse than the reference's Triton path's own error.  The
reference GPU path cannot run here, so this module reproduces its arithmetic
on the CPU:

  * phases 1 and 3 of ``FastWeightMixer.forward`` (train_ablation.py:160-167,
    184-186) under bf16 autocast (train_ablation.py:465-467): every matmul
    rounds its operands to bf16, accumulates in fp32 and rounds its result to
    bf16; elementwise ops follow torch's type promotion (bf16 with fp32 gives
    fp32); the backward of each matmul runs on the bf16 tensors, as autograd
    does under autocast;
  * phase 2 through the Triton kernels' default precision (fast_scan.py:196-199,
    ``tl.dot`` without ``input_precision``, i.e. tf32): every product of the
    scan, forward and backward, Newton-Schulz included, rounds its fp32
    operands to tf32 (10 explicit mantissa bits, round to nearest even) and
    accumulates in fp32, on the pre-update-state recurrence of
    fast_scan.py:72-95 (``Uv.float()``, ``Kw.float()`` in, ``states.to(bf16)``
    out, train_ablation.py:181-185).

The backward of the scan is autograd of the tf32-rounded forward, which uses
the same products as the Triton backward (fast_scan.py:269-331: G recomputed,
``dK = -S^T Gbar``, ``Gbar K^T``, the msign VJP) with the same operand
rounding; it is an emulation of those numerics, not a bit-exact replay.

TEST INFRASTRUCTURE ONLY: used by ``tests/`` as the "reference Triton path's
own error" arm of the bf16 parity bar.
"""

from __future__ import annotations

import torch

from .mixer_oracle import chunk_gate_scalars, token_weights
from .scan_oracle import scan_forward


def round_tf32(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> tf32 (keep 10 mantissa bits, round to nearest even), as fp32."""
    x = x.float().contiguous()
    bits = x.view(torch.int32)
    lsb = (bits >> 13) & 1
    r = (bits + 0x0FFF + lsb) & ~0x1FFF
    finite = torch.isfinite(x)
    return torch.where(finite, r.view(torch.float32), x)


class _Tf32MatMul(torch.autograd.Function):
    """a @ b with tf32 operands and fp32 accumulation, backward likewise."""

    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return round_tf32(a) @ round_tf32(b)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        gt = round_tf32(g)
        return gt @ round_tf32(b).transpose(-1, -2), round_tf32(a).transpose(-1, -2) @ gt


def tf32_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return _Tf32MatMul.apply(a, b)


class _AutocastMatMul(torch.autograd.Function):
    """a @ b as under bf16 autocast: bf16 operands, fp32 accumulation, bf16
    result; the backward multiplies the bf16 cotangent by the bf16 operands and
    rounds each gradient to bf16."""

    @staticmethod
    def forward(ctx, a, b):
        a16 = a.to(torch.bfloat16).float()
        b16 = b.to(torch.bfloat16).float()
        ctx.save_for_backward(a16, b16)
        return (a16 @ b16).to(torch.bfloat16).float()

    @staticmethod
    def backward(ctx, g):
        a16, b16 = ctx.saved_tensors
        g16 = g.to(torch.bfloat16).float()
        ga = (g16 @ b16.transpose(-1, -2)).to(torch.bfloat16).float()
        gb = (a16.transpose(-1, -2) @ g16).to(torch.bfloat16).float()
        return ga, gb


def _amm(a, b):
    return _AutocastMatMul.apply(a, b)


class _RoundBf16(torch.autograd.Function):
    """A bf16 tensor of an elementwise bf16 op (both operands bf16): value and
    cotangent rounded to bf16."""

    @staticmethod
    def forward(ctx, x):
        return x.to(torch.bfloat16).float()

    @staticmethod
    def backward(ctx, g):
        return g.to(torch.bfloat16).float()


def _r16(x):
    return _RoundBf16.apply(x)


def mixer_core_forward(q, k, v, alpha, beta, mu, nu, rule: int, ns: int, chunk: int = 64):
    """o (B, H, T, dh) with the reference's GPU numerics.  q, k, v carry
    bf16-representable values (the trainer's activations are bf16); the gates
    keep the dtype they are given (fp32 here), so products with them promote
    to fp32 exactly as torch does under autocast.  All tensors are fp32
    containers; roundings are explicit."""
    Bsz, H, T, dh = q.shape
    C = chunk
    N = T // C
    qn = _r16(q).reshape(Bsz, H, N, C, dh)
    kn = _r16(k).reshape(Bsz, H, N, C, dh)
    vn = _r16(v).reshape(Bsz, H, N, C, dh)
    an = alpha.reshape(Bsz, H, N, C)
    bn = beta.reshape(Bsz, H, N, C)
    mn = mu.reshape(Bsz, H, N, C)
    nun = nu.reshape(Bsz, H, N, C) if (rule == 2 and nu is not None) else None

    w = token_weights(bn, mn, rule)                       # fp32 (fp32 gates)
    causal = torch.ones(C, C, dtype=torch.bool).tril()
    A = (_amm(qn, kn.transpose(-1, -2)) * bn.unsqueeze(-2)).masked_fill(~causal, 0.0)
    Kw = _amm((kn * w.unsqueeze(-1)).transpose(-1, -2), kn)     # bf16 * fp32 -> fp32 -> mm
    Uv = _amm((vn * w.unsqueeze(-1)).transpose(-1, -2), kn)
    Qt = _r16(qn - _amm(A, kn))                            # bf16 - bf16 -> bf16
    Ov = _amm(A, vn)

    a_c, b_c, m_c, n_c = chunk_gate_scalars(an, bn, mn, nun)
    states = scan_forward(Uv.float(), Kw.float(), a_c, b_c, m_c, n_c, rule, ns, tf32_matmul)
    Sst = _r16(states)                                     # states.to(bf16)
    o = _r16(_amm(Qt, Sst.transpose(-1, -2)) + Ov)         # bf16 + bf16 -> bf16
    return o.reshape(Bsz, H, T, dh)
