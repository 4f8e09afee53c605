"""torch.library custom ops over the C ABI, with autograd and fake (meta) kernels.

Two ops, matching the two layers of the reference they replace:

``state_scan(U, K, a, b, m, n, rule, ns)``
    fast_scan.py:403 ``fast_state_scan`` / ``_TritonScan`` (fast_scan.py:334-396):
    pre-update states (B, H, N, dh, dh) of the chunk recurrence.

``chunk_fast_weight(q, k, v, alpha, beta, mu, nu, rule, ns, chunk)``
    train_ablation.py:142-187 (phases 1-3 of ``FastWeightMixer.forward``):
    o (B, H, T, dh) from q, k, v and the per-token gates.

``mixer_prologue(u, conv_weight, conv_bias, gate_logits, n_heads)``
    train_ablation.py:124-140 after the two projections: q, k, v (B, H, T, dh)
    and the gates (nG, B, H, T).

``head_rmsnorm(o, weight, eps, out_dtype)``
    train_ablation.py:188-189 up to the output projection: the per-head
    RMSNorm of o written as (B, T, H * dh).

Both run only on CUDA tensors through ``libgmdn_b200.so``; there is no CPU or
eager fallback.  The ops are opaque to torch.compile (fake kernels give the
output shapes), so a compiled trainer can call them.
"""

from __future__ import annotations

import ctypes
import os
from typing import Optional

import torch
from torch import Tensor

from ._lib import GMDN_PREC_FAST, GMDN_PREC_IEEE, check, lib

__all__ = ["state_scan", "chunk_fast_weight", "head_rmsnorm", "mixer_prologue",
           "GMDN_PREC_IEEE", "GMDN_PREC_FAST", "ScanFunction"]


def _ptr(t: Optional[Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(None)


def _stream(t: Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _require_cuda(name: str, *tensors: Optional[Tensor]) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                f"{name}: the B200 op runs on CUDA tensors only (got a {t.device} tensor); "
                "this build has no CPU or eager fallback")


def _scratch(nbytes: int, like: Tensor) -> Tensor:
    """An opaque byte buffer (the op's `saved` output).  The kernels fill its
    pieces but never the alignment padding between them, nor the one-byte
    placeholder of a rule that saves nothing; small buffers are zeroed so that
    two calls on the same inputs return equal bytes (torch.library.opcheck
    compares every output), large ones are left as allocated."""
    n = max(int(nbytes), 1)
    alloc = torch.zeros if n <= (1 << 20) else torch.empty
    return alloc(n, dtype=torch.uint8, device=like.device)


# GMDN_CHECK_STATUS=1: after every mixer-core call, synchronise and read the
# kernels' device status word (a bounded wait that gave up raises here).
_CHECK_STATUS = os.environ.get("GMDN_CHECK_STATUS", "0") == "1"


def _check_status(ws: Tensor, what: str) -> None:
    # reading the word synchronises the stream: not while it is being
    # captured into a CUDA graph (the replays are checked by their caller)
    if _CHECK_STATUS and not torch.cuda.is_current_stream_capturing():
        check(lib.gmdn_chunk_status(_ptr(ws), _stream(ws)), what)


# ---------------------------------------------------------------------------
# phase-2 state scan
# ---------------------------------------------------------------------------

@torch.library.custom_op("gmdn::state_scan_fwd", mutates_args=())
def _state_scan_fwd(U: Tensor, K: Tensor, a: Tensor, b: Tensor, m: Tensor, n: Tensor,
                    rule: int, ns: int, precision: int) -> tuple[Tensor, Tensor]:
    B, H, N, dh, _ = U.shape
    S = torch.empty_like(U)
    saved = _scratch(lib.gmdn_scan_saved_bytes(B, H, N, dh, rule), U)
    ws_bytes = lib.gmdn_scan_workspace_bytes(B, H, N, dh, rule, ns, precision)
    ws = _scratch(ws_bytes, U)
    with torch.cuda.device(U.device):
        rc = lib.gmdn_scan_fwd(_ptr(U), _ptr(K), _ptr(a), _ptr(b), _ptr(m), _ptr(n), _ptr(S),
                               _ptr(saved), _ptr(ws), ws_bytes, B, H, N, dh, rule, ns,
                               precision, _stream(U))
    check(rc, "gmdn_scan_fwd")
    if S.numel():
        _check_status(ws, "gmdn_scan_fwd (device)")
    return S, saved


@_state_scan_fwd.register_fake
def _(U, K, a, b, m, n, rule, ns, precision):
    B, H, N, dh, _ = U.shape
    return torch.empty_like(U), U.new_empty(
        max(int(lib.gmdn_scan_saved_bytes(B, H, N, dh, rule)), 1), dtype=torch.uint8)


@torch.library.custom_op("gmdn::state_scan_bwd", mutates_args=())
def _state_scan_bwd(U: Tensor, K: Tensor, a: Tensor, b: Tensor, m: Tensor, n: Tensor,
                    S: Tensor, saved: Tensor, gS: Tensor, rule: int, ns: int,
                    precision: int) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    B, H, N, dh, _ = U.shape
    dU, dK = torch.empty_like(U), torch.empty_like(K)
    da, db, dm, dn = (torch.empty_like(t) for t in (a, b, m, n))
    ws_bytes = lib.gmdn_scan_workspace_bytes(B, H, N, dh, rule, ns, precision)
    ws = _scratch(ws_bytes, U)
    with torch.cuda.device(U.device):
        rc = lib.gmdn_scan_bwd(_ptr(U), _ptr(K), _ptr(a), _ptr(b), _ptr(m), _ptr(n), _ptr(S),
                               _ptr(saved), _ptr(gS), _ptr(dU), _ptr(dK), _ptr(da), _ptr(db),
                               _ptr(dm), _ptr(dn), _ptr(ws), ws_bytes, B, H, N, dh, rule, ns,
                               precision, _stream(U))
    check(rc, "gmdn_scan_bwd")
    if dU.numel():
        _check_status(ws, "gmdn_scan_bwd (device)")
    return dU, dK, da, db, dm, dn


@_state_scan_bwd.register_fake
def _(U, K, a, b, m, n, S, saved, gS, rule, ns, precision):
    return (torch.empty_like(U), torch.empty_like(K), torch.empty_like(a), torch.empty_like(b),
            torch.empty_like(m), torch.empty_like(n))


def _scan_setup(ctx, inputs, output):
    U, K, a, b, m, n, rule, ns, precision = inputs
    S, saved = output
    ctx.save_for_backward(U, K, a, b, m, n, S, saved)
    ctx.cfg = (rule, ns, precision)
    ctx.set_materialize_grads(False)  # never build a zero cotangent for `saved`


def _scan_backward(ctx, gS, _gsaved):
    U, K, a, b, m, n, S, saved = ctx.saved_tensors
    rule, ns, precision = ctx.cfg
    if gS is None:
        gS = torch.zeros_like(S)
    grads = torch.ops.gmdn.state_scan_bwd(U, K, a, b, m, n, S, saved, gS.contiguous(), rule,
                                          ns, precision)
    return (*grads, None, None, None)


_state_scan_fwd.register_autograd(_scan_backward, setup_context=_scan_setup)


def _check_scan_args(U, K, a, b, m, n, rule, ns):
    if U.dim() != 5 or U.shape[-1] != U.shape[-2]:
        raise ValueError(f"U must be (B, H, N, dh, dh) with square states, got {tuple(U.shape)}")
    if K.shape != U.shape:
        raise ValueError(f"K shape {tuple(K.shape)} != U shape {tuple(U.shape)}")
    for name, g in zip("abmn", (a, b, m, n)):
        if g.shape != U.shape[:3]:
            raise ValueError(f"gate {name} must be (B, H, N) = {tuple(U.shape[:3])}, "
                             f"got {tuple(g.shape)}")
    if rule not in (0, 1, 2):
        raise ValueError(f"rule must be 0 (delta), 1 (muon) or 2 (adam), got {rule}")
    if ns < 0:
        raise ValueError(f"ns must be >= 0, got {ns}")


def state_scan(U: Tensor, K: Tensor, a: Tensor, b: Tensor, m: Tensor, n: Tensor, rule: int,
               ns: int, precision: int = GMDN_PREC_IEEE) -> Tensor:
    """Pre-update state stack (B, H, N, dh, dh), differentiable in all six inputs."""
    _check_scan_args(U, K, a, b, m, n, rule, ns)
    _require_cuda("state_scan", U, K, a, b, m, n)
    args = [t.float().contiguous() for t in (U, K, a, b, m, n)]
    S, _ = torch.ops.gmdn.state_scan_fwd(*args, int(rule), int(ns), int(precision))
    return S


class ScanFunction:
    """``_TritonScan``-compatible entry: ``ScanFunction.apply(U, K, a, b, m, n,
    rule, ns)`` (fast_scan.py:334-396), using the precision set in the shim."""

    precision = GMDN_PREC_FAST

    @staticmethod
    def apply(U, K, a, b, m, n, rule, ns):
        return state_scan(U, K, a, b, m, n, rule, ns, ScanFunction.precision)


# ---------------------------------------------------------------------------
# mixer core (phases 1-3)
# ---------------------------------------------------------------------------

def _io_flag(q: Tensor) -> int:
    if q.dtype == torch.bfloat16:
        return 0
    if q.dtype == torch.float32:
        return 1
    raise TypeError(f"q/k/v must be bfloat16 or float32, got {q.dtype}")


@torch.library.custom_op("gmdn::chunk_fwd", mutates_args=())
def _chunk_fwd(q: Tensor, k: Tensor, v: Tensor, alpha: Tensor, beta: Tensor, mu: Tensor,
               nu: Optional[Tensor], rule: int, ns: int, chunk: int,
               precision: int) -> tuple[Tensor, Tensor]:
    B, H, T, dh = q.shape
    io = _io_flag(q)
    o = torch.empty_like(q)
    saved = _scratch(lib.gmdn_chunk_saved_bytes_ex(B, H, T, dh, chunk, rule, ns, precision, io),
                     q)
    ws_bytes = lib.gmdn_chunk_workspace_bytes_ex(B, H, T, dh, chunk, rule, ns, precision, io)
    ws = _scratch(ws_bytes, q)
    with torch.cuda.device(q.device):
        rc = lib.gmdn_chunk_fwd_ex(_ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(beta), _ptr(mu),
                                   _ptr(nu), _ptr(o), _ptr(saved), _ptr(ws), ws_bytes, B, H, T,
                                   dh, chunk, rule, ns, precision, io, _stream(q))
    check(rc, "gmdn_chunk_fwd")
    _check_status(ws, "gmdn_chunk_fwd (device)")
    return o, saved


@_chunk_fwd.register_fake
def _(q, k, v, alpha, beta, mu, nu, rule, ns, chunk, precision):
    B, H, T, dh = q.shape
    nbytes = max(int(lib.gmdn_chunk_saved_bytes_ex(B, H, T, dh, chunk, rule, ns, precision,
                                                   _io_flag(q))), 1)
    return torch.empty_like(q), q.new_empty(nbytes, dtype=torch.uint8)


@torch.library.custom_op("gmdn::chunk_bwd", mutates_args=())
def _chunk_bwd(q: Tensor, k: Tensor, v: Tensor, alpha: Tensor, beta: Tensor, mu: Tensor,
               nu: Optional[Tensor], dO: Tensor, saved: Tensor, rule: int, ns: int, chunk: int,
               precision: int) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    B, H, T, dh = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dalpha, dbeta, dmu = torch.empty_like(alpha), torch.empty_like(beta), torch.empty_like(mu)
    dnu = torch.empty_like(nu) if nu is not None else alpha.new_empty(0)
    io = _io_flag(q)
    ws_bytes = lib.gmdn_chunk_workspace_bytes_ex(B, H, T, dh, chunk, rule, ns, precision, io)
    ws = _scratch(ws_bytes, q)
    with torch.cuda.device(q.device):
        rc = lib.gmdn_chunk_bwd_ex(_ptr(q), _ptr(k), _ptr(v), _ptr(alpha), _ptr(beta), _ptr(mu),
                                   _ptr(nu), _ptr(dO), _ptr(saved), _ptr(dq), _ptr(dk), _ptr(dv),
                                   _ptr(dalpha), _ptr(dbeta), _ptr(dmu),
                                   _ptr(dnu if nu is not None else None), _ptr(ws), ws_bytes,
                                   B, H, T, dh, chunk, rule, ns, precision, io, _stream(q))
    check(rc, "gmdn_chunk_bwd")
    _check_status(ws, "gmdn_chunk_bwd (device)")
    return dq, dk, dv, dalpha, dbeta, dmu, dnu


@_chunk_bwd.register_fake
def _(q, k, v, alpha, beta, mu, nu, dO, saved, rule, ns, chunk, precision):
    dnu = torch.empty_like(nu) if nu is not None else alpha.new_empty(0)
    return (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
            torch.empty_like(alpha), torch.empty_like(beta), torch.empty_like(mu), dnu)


def _chunk_setup(ctx, inputs, output):
    q, k, v, alpha, beta, mu, nu, rule, ns, chunk, precision = inputs
    _, saved = output
    ctx.has_nu = nu is not None
    ctx.save_for_backward(q, k, v, alpha, beta, mu, nu if nu is not None else alpha.new_empty(0),
                          saved)
    ctx.cfg = (rule, ns, chunk, precision)
    ctx.set_materialize_grads(False)  # never build a zero cotangent for `saved`


def _chunk_backward(ctx, dO, _dsaved):
    q, k, v, alpha, beta, mu, nu, saved = ctx.saved_tensors
    if dO is None:
        dO = torch.zeros_like(q)
    nu = nu if ctx.has_nu else None
    rule, ns, chunk, precision = ctx.cfg
    dq, dk, dv, dalpha, dbeta, dmu, dnu = torch.ops.gmdn.chunk_bwd(
        q, k, v, alpha, beta, mu, nu, dO.contiguous(), saved, rule, ns, chunk, precision)
    return dq, dk, dv, dalpha, dbeta, dmu, (dnu if ctx.has_nu else None), None, None, None, None


_chunk_fwd.register_autograd(_chunk_backward, setup_context=_chunk_setup)


def chunk_fast_weight(q: Tensor, k: Tensor, v: Tensor, alpha: Tensor, beta: Tensor,
                      mu: Tensor, nu: Optional[Tensor], rule: int, ns: int, chunk: int = 64,
                      precision: int = GMDN_PREC_FAST) -> Tensor:
    """Phases 1-3 of the reference mixer (train_ablation.py:142-187).

    q, k, v: (B, H, T, dh), bf16 or fp32 (q and k already L2-normalised, as at
    train_ablation.py:127-128).  alpha, beta, mu, nu: (B, H, T) gate values in
    (0, 1); nu is read only by rule 2 (adam).  Returns o (B, H, T, dh) in the
    dtype of q, before the per-head RMSNorm of train_ablation.py:188.
    """
    if q.dim() != 4:
        raise ValueError(f"q must be (B, H, T, dh), got {tuple(q.shape)}")
    B, H, T, dh = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k and v must have the same shape")
    if T % chunk:
        raise ValueError(f"seq_len {T} must be a multiple of the chunk size {chunk}")
    if rule not in (0, 1, 2):
        raise ValueError(f"rule must be 0 (delta), 1 (muon) or 2 (adam), got {rule}")
    if rule == 2 and nu is None:
        raise ValueError("adam (rule 2) needs the nu gate")
    for name, g in (("alpha", alpha), ("beta", beta), ("mu", mu), ("nu", nu)):
        if g is not None and g.shape != (B, H, T):
            raise ValueError(f"gate {name} must be (B, H, T) = {(B, H, T)}, got {tuple(g.shape)}")
    _require_cuda("chunk_fast_weight", q, k, v, alpha, beta, mu, nu)
    dt = q.dtype
    q, k, v = (t.to(dt).contiguous() for t in (q, k, v))
    gates = [g.float().contiguous() if g is not None else None for g in (alpha, beta, mu, nu)]
    if rule != 2:
        gates[3] = None
    o, _ = torch.ops.gmdn.chunk_fwd(q, k, v, *gates, int(rule), int(ns), int(chunk),
                                    int(precision))
    return o


# ---------------------------------------------------------------------------
# mixer epilogue: per-head RMSNorm into the (B, T, D) layout
# ---------------------------------------------------------------------------

def _f32_flag(t: Tensor, what: str) -> int:
    if t.dtype == torch.bfloat16:
        return 0
    if t.dtype == torch.float32:
        return 1
    raise TypeError(f"{what} must be bfloat16 or float32, got {t.dtype}")


def _aligned(t: Tensor) -> Tensor:
    """Contiguous and 16-byte aligned (a fresh copy when a view is not).  Under
    tracing (fake or functional tensors have no storage) only contiguity is
    imposed; the real call that follows checks the alignment."""
    t = t.contiguous()
    try:
        ptr = t.data_ptr()
    except RuntimeError:
        return t
    return t if ptr % 16 == 0 else t.clone()


@torch.library.custom_op("gmdn::head_rmsnorm_fwd", mutates_args=())
def _head_rmsnorm_fwd(o: Tensor, weight: Tensor, eps: float, out_f32: bool) -> Tensor:
    B, H, T, dh = o.shape
    y = torch.empty(B, T, H * dh, dtype=torch.float32 if out_f32 else torch.bfloat16,
                    device=o.device)
    with torch.cuda.device(o.device):
        rc = lib.gmdn_head_rmsnorm_fwd(_ptr(o), _ptr(weight), _ptr(y), B, H, T, dh, float(eps),
                                       _f32_flag(o, "o"), int(out_f32), _stream(o))
    check(rc, "gmdn_head_rmsnorm_fwd")
    return y


@_head_rmsnorm_fwd.register_fake
def _(o, weight, eps, out_f32):
    B, H, T, dh = o.shape
    return o.new_empty(B, T, H * dh, dtype=torch.float32 if out_f32 else torch.bfloat16)


@torch.library.custom_op("gmdn::head_rmsnorm_bwd", mutates_args=())
def _head_rmsnorm_bwd(o: Tensor, weight: Tensor, dy: Tensor, eps: float,
                      out_f32: bool) -> tuple[Tensor, Tensor]:
    B, H, T, dh = o.shape
    d_o = torch.empty_like(o)
    dw = torch.empty(dh, dtype=torch.float32, device=o.device)
    with torch.cuda.device(o.device):
        rc = lib.gmdn_head_rmsnorm_bwd(_ptr(o), _ptr(weight), _ptr(dy), _ptr(d_o), _ptr(dw), B, H,
                                       T, dh, float(eps), _f32_flag(o, "o"), int(out_f32),
                                       _stream(o))
    check(rc, "gmdn_head_rmsnorm_bwd")
    return d_o, dw


@_head_rmsnorm_bwd.register_fake
def _(o, weight, dy, eps, out_f32):
    return torch.empty_like(o), weight.new_empty(o.shape[-1], dtype=torch.float32)


def _rms_setup(ctx, inputs, output):
    o, weight, eps, out_f32 = inputs
    ctx.save_for_backward(o, weight)
    ctx.cfg = (eps, out_f32)
    ctx.weight_dtype = weight.dtype


def _rms_backward(ctx, dy):
    o, weight = ctx.saved_tensors
    eps, out_f32 = ctx.cfg
    dy = _aligned(dy.to(torch.float32 if out_f32 else torch.bfloat16))
    d_o, dw = torch.ops.gmdn.head_rmsnorm_bwd(o, weight, dy, eps, out_f32)
    return d_o, dw, None, None


_head_rmsnorm_fwd.register_autograd(_rms_backward, setup_context=_rms_setup)


def head_rmsnorm(o: Tensor, weight: Tensor, eps: Optional[float] = None,
                 out_dtype: Optional[torch.dtype] = None) -> Tensor:
    """The mixer epilogue before the output projection (train_ablation.py:188-189):
    ``norm(o).to(out_dtype).transpose(1, 2).reshape(B, T, H * dh)`` with
    ``norm = nn.RMSNorm(dh)``.

    o: (B, H, T, dh) bf16 or fp32 (the output of ``chunk_fast_weight``);
    weight: (dh,) the RMSNorm weight; eps: None for torch's default for bf16 /
    fp32 input (float32 machine epsilon); out_dtype: bf16 or fp32, default the
    dtype of o.  Each row is normalised in fp32, rounded to o's dtype and stored
    in out_dtype, as torch's rms_norm followed by ``.to(x.dtype)`` does.
    Returns (B, T, H * dh); differentiable in o and weight.  dh 32, 64 or 128.
    """
    if o.dim() != 4:
        raise ValueError(f"o must be (B, H, T, dh), got {tuple(o.shape)}")
    dh = o.shape[-1]
    if weight.shape != (dh,):
        raise ValueError(f"weight must be ({dh},), got {tuple(weight.shape)}")
    if dh not in (32, 64, 128):
        raise ValueError(f"head_rmsnorm supports dh 32, 64 or 128 (got {dh})")
    _require_cuda("head_rmsnorm", o, weight)
    out_dtype = o.dtype if out_dtype is None else out_dtype
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"out_dtype must be bfloat16 or float32, got {out_dtype}")
    _f32_flag(o, "o")
    e = -1.0 if eps is None else float(eps)
    w = weight.float()   # differentiable; the gradient comes back in weight's dtype
    return torch.ops.gmdn.head_rmsnorm_fwd(_aligned(o), _aligned(w), e,
                                           out_dtype == torch.float32)


# ---------------------------------------------------------------------------
# mixer prologue: conv + SiLU + q/k L2 norm + head layout, gate sigmoids
# ---------------------------------------------------------------------------

@torch.library.custom_op("gmdn::mixer_prologue_fwd", mutates_args=())
def _prologue_fwd(u: Tensor, conv_w: Tensor, conv_b: Tensor, gl: Tensor,
                  n_heads: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    B, T, D3 = u.shape
    H = n_heads
    dh = D3 // 3 // H
    nG = gl.shape[-1] // H
    q = u.new_empty(B, H, T, dh)
    k, v = torch.empty_like(q), torch.empty_like(q)
    g = gl.new_empty(nG, B, H, T)
    with torch.cuda.device(u.device):
        rc = lib.gmdn_mixer_prologue_fwd(_ptr(u), _ptr(conv_w), _ptr(conv_b), _ptr(gl), _ptr(q),
                                         _ptr(k), _ptr(v), _ptr(g), B, T, H, dh, nG,
                                         _f32_flag(u, "u"), _stream(u))
    check(rc, "gmdn_mixer_prologue_fwd")
    return q, k, v, g


@_prologue_fwd.register_fake
def _(u, conv_w, conv_b, gl, n_heads):
    B, T, D3 = u.shape
    dh = D3 // 3 // n_heads
    q = u.new_empty(B, n_heads, T, dh)
    return q, torch.empty_like(q), torch.empty_like(q), gl.new_empty(gl.shape[-1] // n_heads, B,
                                                                      n_heads, T)


@torch.library.custom_op("gmdn::mixer_prologue_bwd", mutates_args=())
def _prologue_bwd(u: Tensor, conv_w: Tensor, conv_b: Tensor, gl: Tensor, dq: Tensor, dk: Tensor,
                  dv: Tensor, dg: Tensor, n_heads: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    B, T, D3 = u.shape
    H = n_heads
    dh = D3 // 3 // H
    nG = gl.shape[-1] // H
    du, dgl = torch.empty_like(u), torch.empty_like(gl)
    dcw = torch.empty(D3, 1, 4, dtype=torch.float32, device=u.device)
    dcb = torch.empty(D3, dtype=torch.float32, device=u.device)
    with torch.cuda.device(u.device):
        rc = lib.gmdn_mixer_prologue_bwd(_ptr(u), _ptr(conv_w), _ptr(conv_b), _ptr(gl), _ptr(dq),
                                         _ptr(dk), _ptr(dv), _ptr(dg), _ptr(du), _ptr(dcw),
                                         _ptr(dcb), _ptr(dgl), B, T, H, dh, nG,
                                         _f32_flag(u, "u"), _stream(u))
    check(rc, "gmdn_mixer_prologue_bwd")
    return du, dcw, dcb, dgl


@_prologue_bwd.register_fake
def _(u, conv_w, conv_b, gl, dq, dk, dv, dg, n_heads):
    D3 = u.shape[-1]
    return (torch.empty_like(u), u.new_empty(D3, 1, 4, dtype=torch.float32),
            u.new_empty(D3, dtype=torch.float32), torch.empty_like(gl))


def _pro_setup(ctx, inputs, output):
    u, conv_w, conv_b, gl, n_heads = inputs
    ctx.save_for_backward(u, conv_w, conv_b, gl)
    ctx.n_heads = n_heads


def _pro_backward(ctx, dq, dk, dv, dg):
    u, conv_w, conv_b, gl = ctx.saved_tensors
    z = lambda t, like: torch.zeros_like(like) if t is None else _aligned(t.to(like.dtype))
    B, T, D3 = u.shape
    H = ctx.n_heads
    dh = D3 // 3 // H
    shape = u.new_empty(B, H, T, dh)
    gshape = gl.new_empty(gl.shape[-1] // H, B, H, T)
    du, dcw, dcb, dgl = torch.ops.gmdn.mixer_prologue_bwd(
        u, conv_w, conv_b, gl, z(dq, shape), z(dk, shape), z(dv, shape), z(dg, gshape), H)
    return du, dcw, dcb, dgl, None


_prologue_fwd.register_autograd(_pro_backward, setup_context=_pro_setup)


def mixer_prologue(u: Tensor, conv_weight: Tensor, conv_bias: Tensor, gate_logits: Tensor,
                   n_heads: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """The mixer prologue after the two projections (train_ablation.py:124-140).

    u = self.qkv(x): (B, T, 3D); conv_weight (3D, 1, 4) and conv_bias (3D,) of
    the depthwise causal Conv1d (kernel 4, padding 3); gate_logits =
    self.gates(x): (B, T, nG * H).  Returns q, k (L2-normalised per head, eps
    1e-12), v, all (B, H, T, dh), and the sigmoid gates (nG, B, H, T) (alpha,
    beta, mu[, nu] = g[0], g[1], g[2][, g[3]]), all in u's dtype.  Computed in fp32; bf16 or fp32 I/O; dh 32, 64 or 128.
    Differentiable in u, both conv parameters and gate_logits.
    """
    if u.dim() != 3 or gate_logits.dim() != 3:
        raise ValueError("u must be (B, T, 3D) and gate_logits (B, T, nG*H)")
    B, T, D3 = u.shape
    if D3 % (3 * n_heads):
        raise ValueError(f"3D = {D3} is not divisible by 3 * n_heads = {3 * n_heads}")
    dh = D3 // 3 // n_heads
    if dh not in (32, 64, 128):
        raise ValueError(f"mixer_prologue supports dh 32, 64 or 128 (got {dh})")
    if gate_logits.shape[:2] != (B, T) or gate_logits.shape[-1] % n_heads or \
            gate_logits.shape[-1] // n_heads not in (3, 4):
        raise ValueError(f"gate_logits must be (B, T, 3 or 4 * H), got {tuple(gate_logits.shape)}")
    if tuple(conv_weight.shape) != (D3, 1, 4) or tuple(conv_bias.shape) != (D3,):
        raise ValueError("conv must be depthwise with kernel 4: weight (3D, 1, 4), bias (3D,)")
    _require_cuda("mixer_prologue", u, conv_weight, conv_bias, gate_logits)
    _f32_flag(u, "u")
    gl = gate_logits.to(u.dtype)
    return torch.ops.gmdn.mixer_prologue_fwd(_aligned(u), _aligned(conv_weight.float()),
                                             _aligned(conv_bias.float()), _aligned(gl),
                                             int(n_heads))
