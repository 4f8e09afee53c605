"""Helpers that run the CPU oracle for the GPU parity tests."""
import torch

import oracle


def scan_oracle(base, gS, rule, ns, dtype):
    """Forward states and the six cotangents from the oracle in `dtype`."""
    ins = [t.detach().to(dtype) for t in base]
    S, M, V = oracle.scan_forward_all(*ins, rule, ns)
    grads = oracle.scan_backward(*ins, S, M, V, gS.to(dtype), rule, ns)
    return S, list(grads)


def mixer_oracle(inp, rule, ns, chunk, dtype):
    """o and the cotangents of q, k, v, alpha, beta, mu, nu from autograd of the
    oracle mixer core, evaluated in `dtype` on the given (already rounded) inputs."""
    names = ["q", "k", "v", "alpha", "beta", "mu", "nu"]
    ins = []
    for n in names:
        t = getattr(inp, n)
        ins.append(None if t is None else t.detach().to(dtype).requires_grad_(True))
    o = oracle.mixer_core_forward(*ins, rule, ns, chunk)
    (o * inp.dO.detach().to(dtype)).sum().backward()
    grads = {}
    for n, t in zip(names, ins):
        if t is not None:
            grads["d" + n] = t.grad if t.grad is not None else torch.zeros_like(t)
    return o.detach(), grads
