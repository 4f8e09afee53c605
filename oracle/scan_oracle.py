"""CPU restatement of the reference's fast-weight state scan (TEST ORACLE).

Reference: ``fast_scan.py`` of cloud-777-boy/GMDN-GATED-MUON-DELTANET.

  * the recurrence and constants   -- fast_scan.py:5-15, 32-34
  * forward (``scan_eager``)         -- fast_scan.py:72-95
  * Newton-Schulz msign             -- fast_scan.py:63-69
  * hand-derived reverse scan       -- fast_scan.py:134-186
  * msign VJP                       -- fast_scan.py:107-131

Everything here runs in whatever floating type the inputs carry (fp32 for the
"naive fp32 recurrence" the parity bar is stated against, fp64 as ground
truth).  The functions are written without in-place updates so that torch
autograd can differentiate ``scan_forward`` as a second, independent check of
``scan_backward``.

Conventions (same as the reference): U, K are (B, H, N, dh, dh); the gates a,
b, m, n are (B, H, N); each state is stored [dv, dk] (rows = value dim); the
scan returns the PRE-update states S_0 .. S_{N-1}.
"""

from __future__ import annotations

import torch

# Quintic Newton-Schulz coefficients and the two epsilons (fast_scan.py:32-34).
NS_COEF = (3.4445, -4.7750, 2.0315)
EPS_NORM = 1e-7
EPS_ADAM = 1e-6


def _fro(x: torch.Tensor) -> torch.Tensor:
    """Frobenius norm over the two trailing dims, kept for broadcasting."""
    return x.square().sum(dim=(-2, -1), keepdim=True).sqrt()


def _ns_iter(x: torch.Tensor, mm=torch.matmul) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """One quintic NS step; returns (x_next, gram, poly) where gram = x x^T and
    poly = c1*gram + c2*gram^2 (fast_scan.py:67-68).  ``mm`` is the matrix
    product (a rounding emulation may replace it)."""
    c0, c1, c2 = NS_COEF
    gram = mm(x, x.transpose(-1, -2))
    poly = c1 * gram + c2 * mm(gram, gram)
    return c0 * x + mm(poly, x), gram, poly


def msign_square(M: torch.Tensor, ns: int, mm=torch.matmul) -> torch.Tensor:
    """Frobenius-normalise, then ``ns`` NS steps (fast_scan.py:63-69)."""
    x = M / (_fro(M) + EPS_NORM)
    for _ in range(ns):
        x, _, _ = _ns_iter(x, mm)
    return x


def msign_square_vjp(M: torch.Tensor, Ybar: torch.Tensor, ns: int) -> torch.Tensor:
    """Cotangent of M for Y = msign_square(M, ns) (fast_scan.py:107-131).

    Unlike the reference (which recomputes the NS chain O(ns^2) times), the
    iterates are kept from one forward pass; the arithmetic per step is the
    same: with G = X X^T and P = c1 G + c2 G^2,
        Bbar = Xbar' X^T,  Gbar = c1 Bbar + c2 (Bbar G + G Bbar),
        Xbar = c0 Xbar' + P Xbar' + (Gbar + Gbar^T) X.
    """
    c0, c1, c2 = NS_COEF
    fro = _fro(M)
    den = fro + EPS_NORM
    xs, grams, polys = [M / den], [], []
    for _ in range(ns):
        nx, g, p = _ns_iter(xs[-1])
        grams.append(g)
        polys.append(p)
        xs.append(nx)
    xbar = Ybar
    for k in reversed(range(ns)):
        x, g, p = xs[k], grams[k], polys[k]
        bbar = xbar @ x.transpose(-1, -2)
        gbar = c1 * bbar + c2 * (bbar @ g + g @ bbar)
        xbar = c0 * xbar + p @ xbar + (gbar + gbar.transpose(-1, -2)) @ x
    inner = (xbar * M).sum(dim=(-2, -1), keepdim=True)
    return xbar / den - inner / den.square() * (M / fro.clamp_min(1e-12))


def _gate(t: torch.Tensor, i: int) -> torch.Tensor:
    return t[:, :, i, None, None]


def _step(rule: int, ns: int, S, M, V, Ui, Ki, ai, bi, mi, ni, mm=torch.matmul):
    """One chunk of the recurrence (fast_scan.py:82-94). Returns (S', M', V')."""
    G = Ui - mm(S, Ki)
    if rule == 0:
        return ai * S + G, M, V
    if rule == 1:
        M1 = mi * M + G
        return ai * S + bi * msign_square(M1, ns, mm), M1, V
    M1 = mi * M + (1 - mi) * G
    V1 = ni * V + (1 - ni) * G.square()
    return ai * S + bi * M1 / (V1.sqrt() + EPS_ADAM), M1, V1


def scan_forward_all(U, K, a, b, m, n, rule: int, ns: int, mm=torch.matmul):
    """Pre-update S, M, V for every chunk, each (B, H, N, dh, dh)."""
    if rule not in (0, 1, 2):
        raise ValueError(f"rule must be 0 (delta), 1 (muon) or 2 (adam), got {rule}")
    Bsz, H, N, dv, dk = U.shape
    S = U.new_zeros(Bsz, H, dv, dk)
    M = torch.zeros_like(S)
    V = torch.zeros_like(S)
    s_hist, m_hist, v_hist = [], [], []
    for i in range(N):
        s_hist.append(S)
        m_hist.append(M)
        v_hist.append(V)
        S, M, V = _step(rule, ns, S, M, V, U[:, :, i], K[:, :, i], _gate(a, i),
                        _gate(b, i), _gate(m, i), _gate(n, i), mm)
    return (torch.stack(s_hist, 2), torch.stack(m_hist, 2), torch.stack(v_hist, 2))


def scan_forward(U, K, a, b, m, n, rule: int, ns: int, mm=torch.matmul) -> torch.Tensor:
    """Pre-update state stack (B, H, N, dh, dh); differentiable by autograd."""
    return scan_forward_all(U, K, a, b, m, n, rule, ns, mm)[0]


def scan_final_state(U, K, a, b, m, n, rule: int, ns: int) -> torch.Tensor:
    """Post-update state S_N after the last chunk (B, H, dh, dh)."""
    Bsz, H, N, dv, dk = U.shape
    S = U.new_zeros(Bsz, H, dv, dk)
    M = torch.zeros_like(S)
    V = torch.zeros_like(S)
    for i in range(N):
        S, M, V = _step(rule, ns, S, M, V, U[:, :, i], K[:, :, i], _gate(a, i),
                        _gate(b, i), _gate(m, i), _gate(n, i))
    return S


def scan_backward(U, K, a, b, m, n, S_all, M_all, V_all, gS, rule: int, ns: int):
    """Reverse scan given the pre-update histories (fast_scan.py:134-186).

    Returns (dU, dK, da, db, dm, dn).  Gates that a rule does not read get
    exact zeros (delta: db, dm, dn; muon: dn), which is what autograd of the
    forward gives and what the reference's eager path returns.
    """
    Bsz, H, N, dv, dk = U.shape
    dU = torch.zeros_like(U)
    dK = torch.zeros_like(K)
    da, db, dm, dn = (torch.zeros_like(t) for t in (a, b, m, n))
    Sbar = U.new_zeros(Bsz, H, dv, dk)  # cotangent of S_{i+1}
    Mbar = torch.zeros_like(Sbar)       # cotangent of M_{i+1}
    Vbar = torch.zeros_like(Sbar)       # cotangent of V_{i+1}
    for i in range(N - 1, -1, -1):
        S = S_all[:, :, i]
        Ki = K[:, :, i]
        ai, bi, mi, ni = (_gate(t, i) for t in (a, b, m, n))
        G = U[:, :, i] - S @ Ki
        da[:, :, i] = (Sbar * S).sum(dim=(-2, -1))
        if rule == 0:
            Gbar = Sbar
        elif rule == 1:
            Mprev = M_all[:, :, i]
            Mi = mi * Mprev + G
            db[:, :, i] = (Sbar * msign_square(Mi, ns)).sum(dim=(-2, -1))
            Mtot = Mbar + msign_square_vjp(Mi, bi * Sbar, ns)
            dm[:, :, i] = (Mtot * Mprev).sum(dim=(-2, -1))
            Mbar = mi * Mtot
            Gbar = Mtot
        else:
            Mprev, Vprev = M_all[:, :, i], V_all[:, :, i]
            G2 = G.square()
            Mi = mi * Mprev + (1 - mi) * G
            Vi = ni * Vprev + (1 - ni) * G2
            root = Vi.sqrt()
            den = root + EPS_ADAM
            db[:, :, i] = (Sbar * (Mi / den)).sum(dim=(-2, -1))
            ub = bi * Sbar
            Mtot = Mbar + ub / den
            Vtot = Vbar - ub * Mi / den.square() / (2 * root.clamp_min(1e-12))
            dm[:, :, i] = (Mtot * (Mprev - G)).sum(dim=(-2, -1))
            dn[:, :, i] = (Vtot * (Vprev - G2)).sum(dim=(-2, -1))
            Mbar = mi * Mtot
            Vbar = ni * Vtot
            Gbar = (1 - mi) * Mtot + 2 * (1 - ni) * G * Vtot
        dU[:, :, i] = Gbar
        dK[:, :, i] = -(S.transpose(-1, -2) @ Gbar)
        Sbar = ai * Sbar - Gbar @ Ki.transpose(-1, -2) + gS[:, :, i]
    return dU, dK, da, db, dm, dn
