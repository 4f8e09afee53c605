"""Tolerance rule shared by the parity tests.

For every output and gradient:
    err(kernel, fp32 oracle) <= max(tol, 4 * err(fp32 oracle, fp64 oracle))
with err = max|x - y| / max|y| (the metric of the reference's test.py:24-25)
and tol = 1e-4 for fp32 inputs, 2e-2 for bf16 inputs.  The second term is the
conditioning floor of the problem itself: where even an fp32 evaluation of the
reference recurrence is that far from fp64 (adam's 1/(2 sqrt V) spikes, muon's
NS chain), no fp32 kernel can do better, the reference's own included.
Gradients that are exactly zero in the oracle (gates a rule never reads) must
be exactly zero in the kernel.
"""
import torch

TOL_FP32 = 1e-4
TOL_BF16 = 2e-2


def rel(x: torch.Tensor, y: torch.Tensor) -> float:
    x = x.detach().double().cpu()
    y = y.detach().double().cpu()
    return (x - y).abs().max().item() / (y.abs().max().item() + 1e-30)


def check(name: str, got, ref32, ref64, tol: float, report: list | None = None) -> None:
    got = got.detach().cpu()
    if ref64.abs().max().item() == 0.0:
        assert got.abs().max().item() == 0.0, f"{name}: expected exact zeros"
        return
    assert torch.isfinite(got).all(), f"{name}: non-finite values"
    floor = rel(ref32, ref64)
    bound = max(tol, 4.0 * floor)
    err = rel(got, ref32)
    if report is not None:
        report.append((name, err, bound, rel(got, ref64), floor))
    assert err <= bound, (f"{name}: rel err {err:.3e} vs fp32 oracle > bound {bound:.3e} "
                          f"(fp32-vs-fp64 floor {floor:.3e}, kernel-vs-fp64 {rel(got, ref64):.3e})")
