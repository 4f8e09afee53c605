"""Hooks that put the B200 ops under the reference's own modules.

``patch_reference(fast_scan_module)``
    Swap only the kernel class of a loaded reference ``fast_scan`` module:
    its ``_TritonScan`` (fast_scan.py:334-396) becomes the B200 op and
    ``HAS_TRITON`` becomes True.  The reference's dispatcher
    (fast_scan.py:403-414), knobs and eager functions stay as they are, so
    ``train_ablation.py --scan auto`` and ``test.py`` run the B200 kernels
    unmodified.

``patch_mixer(FastWeightMixer)``
    Replace ``FastWeightMixer.forward`` (train_ablation.py:111-190) with one
    that keeps the module's own projections and output projection (plain
    GEMMs), runs the conv / SiLU / q-k norm / gate sigmoids (lines 124-140) as
    the fused ``mixer_prologue`` op, phases 1-3 (lines 142-187) as the fused
    ``chunk_fast_weight`` op and the per-head RMSNorm with its (B, T, D) view
    (lines 188-189) as the fused ``head_rmsnorm`` op (dh 32, 64 or 128 and the
    module's own conv shape; otherwise the module's own layers run those
    lines).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ops

_RULES = {"delta": 0, "muon": 1, "adam": 2}


def patch_reference(fast_scan_module):
    mod = fast_scan_module

    class _B200Scan:
        @staticmethod
        def apply(U, K, a, b, m, n, rule, ns):
            prec = ops.GMDN_PREC_IEEE if mod._PRECISION == "ieee" else ops.GMDN_PREC_FAST
            return ops.state_scan(U, K, a, b, m, n, rule, ns, prec)

    mod._TritonScan = _B200Scan
    mod.HAS_TRITON = True
    return mod


def mixer_forward(self, x: torch.Tensor) -> torch.Tensor:
    """FastWeightMixer.forward with phases 1-3 on the B200 op."""
    B, T, D = x.shape
    C, H, dh = self.chunk, self.h, self.dh
    if T % C:
        raise ValueError("seq_len must be a multiple of chunk size")
    u, gl = self.qkv(x), self.gates(x)
    conv = self.conv
    if (dh in (32, 64, 128) and u.dtype in (torch.bfloat16, torch.float32)
            and tuple(conv.kernel_size) == (4,) and tuple(conv.padding) == (3,)
            and conv.groups == conv.in_channels == conv.out_channels == 3 * D
            and conv.bias is not None and self.n_gates in (3, 4)):
        q, k, v, g = ops.mixer_prologue(u, conv.weight, conv.bias, gl, H)
    else:
        qkv = conv(u.transpose(1, 2))[..., :T].transpose(1, 2)
        q, k, v = F.silu(qkv).chunk(3, dim=-1)
        q = F.normalize(q.reshape(B, T, H, dh).transpose(1, 2), dim=-1)
        k = F.normalize(k.reshape(B, T, H, dh).transpose(1, 2), dim=-1)
        v = v.reshape(B, T, H, dh).transpose(1, 2)
        g = torch.sigmoid(gl).view(B, T, self.n_gates, H).permute(2, 0, 3, 1)
    nu = g[3] if self.n_gates == 4 else None
    if not torch.compiler.is_compiling():
        self.last_gate_means = {
            "alpha": g[0].detach().mean(), "beta": g[1].detach().mean(),
            "mu": g[2].detach().mean(),
            "nu": nu.detach().mean() if nu is not None else float("nan"),
        }
    dt = q.dtype if q.dtype in (torch.bfloat16, torch.float32) else torch.float32
    prec = getattr(self, "b200_precision", ops.GMDN_PREC_FAST)
    o = ops.chunk_fast_weight(q.to(dt), k.to(dt), v.to(dt), g[0], g[1], g[2], nu,
                              _RULES[self.inner], self.ns_steps, C, prec)
    norm = self.norm
    if (isinstance(norm, torch.nn.RMSNorm) and norm.weight is not None and dh in (32, 64, 128)
            and x.dtype in (torch.bfloat16, torch.float32)):
        return self.out(ops.head_rmsnorm(o, norm.weight, norm.eps, x.dtype))
    o = norm(o).to(x.dtype)
    return self.out(o.transpose(1, 2).reshape(B, T, D))


def patch_mixer(mixer_cls):
    mixer_cls.forward = mixer_forward
    return mixer_cls
