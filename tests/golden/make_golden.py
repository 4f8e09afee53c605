"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in the development container, where the reference checkout is readable:

    python tests/golden/make_golden.py --ref <path-to-reference-checkout>

It imports the reference's own ``fast_scan.py`` and ``train_ablation.py``
unmodified and records, in float64 on CPU:

  * scan.pt  -- ``fast_scan.scan_eager`` outputs (fast_scan.py:72-95) and the
    autograd gradients for a seeded cotangent, plus ``manual_backward``
    (fast_scan.py:134-186) on the same cases, for rules 0/1/2 and several ns.
  * mixer.pt -- ``FastWeightMixer.forward`` phases 1-3 (train_ablation.py:142-187)
    on seeded activations: the q, k, v and gates that the reference computes
    internally are captured, and the output o (with the RMSNorm and output
    projection replaced by identities) and the gradients of <o, dO> with
    respect to q, k, v and each gate are recorded.

The fixtures are small (dh 16-32, a handful of chunks) so they can be
committed; the GPU box never needs the reference.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def make_scan_inputs(gen, B, H, N, dh, C=16, family="test"):
    """Seeded scan inputs.  family='test' follows the reference test fixture
    shape (test.py:28-38: normalised k, v/sqrt(dh), w in [0, 0.3), gates in
    narrow ranges); family='wide' draws gates from the full (0, 1) range."""
    dt = torch.float64
    k = torch.nn.functional.normalize(torch.randn(B, H, N, C, dh, generator=gen, dtype=dt), dim=-1)
    v = torch.randn(B, H, N, C, dh, generator=gen, dtype=dt) / dh ** 0.5
    w = torch.rand(B, H, N, C, generator=gen, dtype=dt) * 0.3
    K = (k * w.unsqueeze(-1)).mT @ k
    U = (v * w.unsqueeze(-1)).mT @ k
    if family == "test":
        ranges = ((0.2, 0.75), (0.5, 0.2), (0.5, 0.3), (0.2, 0.7))
        gates = [torch.rand(B, H, N, generator=gen, dtype=dt) * r + o for r, o in ranges]
    else:
        gates = [torch.rand(B, H, N, generator=gen, dtype=dt) * 0.98 + 0.01 for _ in range(4)]
    return [U, K] + gates


def scan_cases(fast_scan):
    cases = []
    specs = [
        # (name, rule, ns, family, B, H, N, dh)
        ("delta_test", 0, 3, "test", 1, 2, 4, 16),
        ("delta_wide", 0, 0, "wide", 2, 1, 3, 16),
        ("muon_ns0", 1, 0, "test", 1, 2, 3, 16),
        ("muon_ns3", 1, 3, "test", 1, 2, 4, 16),
        ("muon_ns5", 1, 5, "test", 1, 2, 3, 16),
        ("muon_ns5_wide", 1, 5, "wide", 1, 1, 3, 32),
        ("adam_test", 2, 3, "test", 1, 2, 4, 16),
        ("adam_wide", 2, 0, "wide", 2, 1, 3, 16),
    ]
    for idx, (name, rule, ns, family, B, H, N, dh) in enumerate(specs):
        gen = torch.Generator().manual_seed(1000 + idx)
        base = make_scan_inputs(gen, B, H, N, dh, family=family)
        ins = [t.clone().requires_grad_(True) for t in base]
        S = fast_scan.scan_eager(*ins, rule, ns)
        gS = torch.randn(S.shape, generator=gen, dtype=S.dtype)
        torch.autograd.backward(S, gS)
        grads = [t.grad.detach().clone() if t.grad is not None else torch.zeros_like(t)
                 for t in ins]
        # manual_backward needs the pre-update M and V histories; rebuild them
        # with the reference's own forward step by step.
        with torch.no_grad():
            U, K, a, b, m, n = base
            Mh, Vh = [], []
            Sx = U.new_zeros(B, H, dh, dh)
            Mx = torch.zeros_like(Sx)
            Vx = torch.zeros_like(Sx)
            for i in range(N):
                Mh.append(Mx)
                Vh.append(Vx)
                G = U[:, :, i] - Sx @ K[:, :, i]
                ai = a[:, :, i, None, None]
                if rule == 0:
                    Sx = ai * Sx + G
                elif rule == 1:
                    Mx = m[:, :, i, None, None] * Mx + G
                    Sx = ai * Sx + b[:, :, i, None, None] * fast_scan._msign_sq(Mx, ns)
                else:
                    mi = m[:, :, i, None, None]
                    ni = n[:, :, i, None, None]
                    Mx = mi * Mx + (1 - mi) * G
                    Vx = ni * Vx + (1 - ni) * G.square()
                    Sx = ai * Sx + b[:, :, i, None, None] * Mx / (Vx.sqrt() + fast_scan._EPS_ADAM)
            M_all = torch.stack(Mh, 2)
            V_all = torch.stack(Vh, 2)
            manual = fast_scan.manual_backward(U, K, a, b, m, n, S.detach(), M_all, V_all,
                                               gS, rule, ns)
        cases.append(dict(
            name=name, rule=rule, ns=ns,
            U=base[0], K=base[1], a=base[2], b=base[3], m=base[4], n=base[5],
            gS=gS, S=S.detach(), M_all=M_all, V_all=V_all,
            dU=grads[0], dK=grads[1], da=grads[2], db=grads[3], dm=grads[4], dn=grads[5],
            manual=list(manual),
        ))
    return cases


class _Recorder:
    """Attribute proxy around a module; named functions record their outputs."""

    def __init__(self, inner, names):
        self._inner = inner
        self._names = set(names)
        self.records: dict[str, list] = {n: [] for n in names}

    def __getattr__(self, item):
        fn = getattr(self._inner, item)
        if item not in self._names:
            return fn

        def wrapped(*args, **kwargs):
            out = fn(*args, **kwargs)
            if out.requires_grad:
                out.retain_grad()
            self.records[item].append(out)
            return out
        return wrapped


def mixer_cases(train_ablation, fast_scan):
    fast_scan.set_backend("eager")
    cases = []
    specs = [
        # (name, inner, ns, d_model, heads, T, chunk, B)
        ("delta_c64", "delta", 3, 32, 2, 128, 64, 1),
        ("delta_c32_dh32", "delta", 3, 64, 2, 64, 32, 1),
        ("muon_c32_ns3", "muon", 3, 32, 2, 96, 32, 1),
        ("muon_c64_ns5", "muon", 5, 32, 2, 128, 64, 1),
        ("adam_c32", "adam", 3, 32, 2, 96, 32, 1),
        ("adam_c64", "adam", 3, 16, 1, 128, 64, 2),
    ]
    real_F, real_torch = train_ablation.F, train_ablation.torch
    try:
        for idx, (name, inner, ns, D, H, T, C, B) in enumerate(specs):
            torch.manual_seed(2000 + idx)
            mixer = train_ablation.FastWeightMixer(D, H, inner, chunk=C, ns_steps=ns).double()
            mixer.norm = torch.nn.Identity()
            mixer.out = torch.nn.Identity()
            gen = torch.Generator().manual_seed(3000 + idx)
            x = torch.randn(B, T, D, generator=gen, dtype=torch.float64)
            rf = _Recorder(real_F, ["normalize", "silu"])
            rt = _Recorder(real_torch, ["sigmoid"])
            train_ablation.F, train_ablation.torch = rf, rt
            y = mixer(x)
            train_ablation.F, train_ablation.torch = real_F, real_torch
            dh = D // H
            o = y.view(B, T, H, dh).transpose(1, 2)
            dO = torch.randn(o.shape, generator=gen, dtype=o.dtype)
            (o * dO).sum().backward()
            q, k = rf.records["normalize"]
            silu_out = rf.records["silu"][0]
            g = rt.records["sigmoid"][0]
            nG = mixer.n_gates
            v = silu_out.chunk(3, dim=-1)[2].reshape(B, T, H, dh).transpose(1, 2)
            dv = silu_out.grad.chunk(3, dim=-1)[2].reshape(B, T, H, dh).transpose(1, 2)
            gp = g.detach().view(B, T, nG, H).permute(2, 0, 3, 1)
            dgp = g.grad.view(B, T, nG, H).permute(2, 0, 3, 1)
            case = dict(
                name=name, rule={"delta": 0, "muon": 1, "adam": 2}[inner], ns=ns, chunk=C,
                q=q.detach().contiguous(), k=k.detach().contiguous(), v=v.detach().contiguous(),
                alpha=gp[0].contiguous(), beta=gp[1].contiguous(), mu=gp[2].contiguous(),
                nu=gp[3].contiguous() if nG == 4 else None,
                dO=dO.contiguous(), o=o.detach().contiguous(),
                dq=q.grad.contiguous(), dk=k.grad.contiguous(), dv=dv.contiguous(),
                dalpha=dgp[0].contiguous(), dbeta=dgp[1].contiguous(), dmu=dgp[2].contiguous(),
                dnu=dgp[3].contiguous() if nG == 4 else None,
            )
            cases.append(case)
    finally:
        train_ablation.F, train_ablation.torch = real_F, real_torch
    return cases


def epilogue_cases(train_ablation):
    """train_ablation.py:188-189 on the reference module's own RMSNorm: the norm,
    the dtype conversion to x.dtype and the (B, T, D) view, with autograd."""
    cases = []
    specs = [
        # (name, D, heads, B, T, o dtype, x dtype)
        ("f64_dh32", 64, 2, 2, 8, torch.float64, torch.float64),
        ("f32_dh64", 128, 2, 2, 16, torch.float32, torch.float32),
        ("f32_dh128", 256, 2, 2, 16, torch.float32, torch.float32),
        ("bf16_to_f32_dh128", 256, 2, 2, 16, torch.bfloat16, torch.float32),
        ("bf16_dh64", 128, 2, 1, 16, torch.bfloat16, torch.bfloat16),
    ]
    for idx, (name, D, H, B, T, odt, xdt) in enumerate(specs):
        torch.manual_seed(4000 + idx)
        mixer = train_ablation.FastWeightMixer(D, H, "delta", chunk=8)
        norm = mixer.norm.to(torch.float64 if odt == torch.float64 else torch.float32)
        dh = D // H
        gen = torch.Generator().manual_seed(5000 + idx)
        with torch.no_grad():
            norm.weight.copy_(1.0 + 0.5 * torch.randn(dh, generator=gen, dtype=norm.weight.dtype))
        scale = torch.exp(torch.randn(B, H, T, 1, generator=gen, dtype=torch.float64))
        o = (torch.randn(B, H, T, dh, generator=gen, dtype=torch.float64) * scale).to(odt)
        o.requires_grad_(True)
        y = norm(o).to(xdt)                          # train_ablation.py:188
        y = y.transpose(1, 2).reshape(B, T, D)       # train_ablation.py:189
        dy = torch.randn(y.shape, generator=gen, dtype=torch.float64).to(xdt)
        (y.double() * dy.double()).sum().backward()
        cases.append(dict(name=name, o=o.detach(), weight=norm.weight.detach().clone(),
                          out_dtype=xdt, y=y.detach(), dy=dy, d_o=o.grad.detach(),
                          dweight=norm.weight.grad.detach().clone()))
    return cases


def prologue_cases(train_ablation, fast_scan):
    """train_ablation.py:124-140 inside the reference module's own forward: the
    projections' outputs u = qkv(x) and gl = gates(x) and the conv parameters
    are recorded with forward hooks, the outputs q, k (F.normalize), the SiLU
    output (v part) and the sigmoid gates with the attribute proxies, and all
    their gradients from a backward through the rest of the mixer."""
    fast_scan.set_backend("eager")
    cases = []
    specs = [
        # (name, inner, D, heads, T, chunk, B, dtype)
        ("f64_delta_dh32", "delta", 64, 2, 64, 32, 1, torch.float64),
        ("f32_adam_dh64", "adam", 128, 2, 64, 32, 2, torch.float32),
        ("f32_delta_dh128", "delta", 256, 2, 64, 64, 1, torch.float32),
    ]
    real_F, real_torch = train_ablation.F, train_ablation.torch
    try:
        for idx, (name, inner, D, H, T, C, B, dt) in enumerate(specs):
            torch.manual_seed(6000 + idx)
            mixer = train_ablation.FastWeightMixer(D, H, inner, chunk=C, ns_steps=3).to(dt)
            mixer.norm = torch.nn.Identity()
            mixer.out = torch.nn.Identity()
            rec = {}

            def hook(name_):
                def fn(_mod, _inp, out):
                    out.retain_grad()
                    rec[name_] = out
                return fn
            h1 = mixer.qkv.register_forward_hook(hook("u"))
            h2 = mixer.gates.register_forward_hook(hook("gl"))
            gen = torch.Generator().manual_seed(7000 + idx)
            x = torch.randn(B, T, D, generator=gen, dtype=dt)
            rf = _Recorder(real_F, ["normalize", "silu"])
            rt = _Recorder(real_torch, ["sigmoid"])
            train_ablation.F, train_ablation.torch = rf, rt
            y = mixer(x)
            train_ablation.F, train_ablation.torch = real_F, real_torch
            h1.remove()
            h2.remove()
            dy = torch.randn(y.shape, generator=gen, dtype=dt)
            (y * dy).sum().backward()
            dh = D // H
            q, k = rf.records["normalize"]
            s = rf.records["silu"][0]
            g = rt.records["sigmoid"][0]
            nG = mixer.n_gates
            v = s.chunk(3, dim=-1)[2].reshape(B, T, H, dh).transpose(1, 2)
            dv = s.grad.chunk(3, dim=-1)[2].reshape(B, T, H, dh).transpose(1, 2)
            cases.append(dict(
                name=name, n_heads=H,
                u=rec["u"].detach(), gl=rec["gl"].detach(),
                conv_w=mixer.conv.weight.detach().clone(), conv_b=mixer.conv.bias.detach().clone(),
                q=q.detach().contiguous(), k=k.detach().contiguous(), v=v.detach().contiguous(),
                g=g.detach().view(B, T, nG, H).permute(2, 0, 3, 1).contiguous(),
                dq=q.grad.contiguous(), dk=k.grad.contiguous(), dv=dv.contiguous(),
                dg=g.grad.view(B, T, nG, H).permute(2, 0, 3, 1).contiguous(),
                du=rec["u"].grad.detach(), dgl=rec["gl"].grad.detach(),
                dconv_w=mixer.conv.weight.grad.detach().clone(),
                dconv_b=mixer.conv.bias.grad.detach().clone(),
            ))
    finally:
        train_ablation.F, train_ablation.torch = real_F, real_torch
    return cases


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--which", default="all", choices=["all", "epilogue", "prologue"],
                    help="epilogue / prologue: write only that fixture file")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.ref))
    import fast_scan  # noqa: E402  (the reference's module)
    import train_ablation  # noqa: E402

    torch.set_num_threads(4)
    meta = dict(torch=str(torch.__version__), source="reference fast_scan.py / train_ablation.py, float64 CPU")
    if args.which in ("all", "prologue"):
        pro = prologue_cases(train_ablation, fast_scan)
        torch.save(dict(meta=dict(torch=str(torch.__version__),
                                  source="reference train_ablation.py:124-140 (its own forward), CPU"),
                        cases=pro), os.path.join(args.out, "prologue.pt"))
        print(f"wrote {len(pro)} prologue cases to {args.out}")
        if args.which == "prologue":
            return
    epi = epilogue_cases(train_ablation)
    torch.save(dict(meta=dict(torch=str(torch.__version__),
                              source="reference train_ablation.py:188-189 (its nn.RMSNorm), CPU"),
                    cases=epi), os.path.join(args.out, "epilogue.pt"))
    print(f"wrote {len(epi)} epilogue cases to {args.out}")
    if args.which == "epilogue":
        return
    scan = scan_cases(fast_scan)
    torch.save(dict(meta=meta, cases=scan), os.path.join(args.out, "scan.pt"))
    mixer = mixer_cases(train_ablation, fast_scan)
    torch.save(dict(meta=meta, cases=mixer), os.path.join(args.out, "mixer.pt"))
    print(f"wrote {len(scan)} scan cases and {len(mixer)} mixer cases to {args.out}")


if __name__ == "__main__":
    main()
