"""Drop-in replacement for the reference module ``fast_scan`` (fast_scan.py).

Same public names and argument meaning as the reference:

  * ``fast_state_scan(U, K, a, b, m, n, rule, ns)``   fast_scan.py:403-414
  * ``_TritonScan.apply(U, K, a, b, m, n, rule, ns)``  fast_scan.py:334-396
  * ``set_backend(name)`` / ``set_precision(name)``   fast_scan.py:47-56
  * ``HAS_TRITON``, ``NS_A/NS_B/NS_C``, ``_EPS_NORM``, ``_EPS_ADAM``

Differences, all deliberate:

  * the kernels are the B200 library, not Triton; ``HAS_TRITON`` means "the B200
    op can run here" (a CUDA device is visible);
  * there is no eager/CPU path: CPU tensors, or ``set_backend('eager')``, raise
    RuntimeError instead of falling back (the reference's eager functions
    ``scan_eager`` / ``manual_backward`` are not shipped; keep the reference
    module for them, or use ``patch_reference`` to swap only the kernel class);
  * gradients of gates a rule does not read are zeros (the reference's Triton
    backward returns uninitialised memory there, fast_scan.py:386-389).
"""

from __future__ import annotations

import importlib
import os
import sys

import torch

_PKG_NAME = "gmdn-gated-muon-deltanet_b200"
if __package__:
    _ops = importlib.import_module(".ops", __package__)
else:  # imported as a top-level module with the package directory on sys.path
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    _ops = importlib.import_module(_PKG_NAME + ".ops")

NS_A, NS_B, NS_C = 3.4445, -4.7750, 2.0315
_EPS_NORM = 1e-7
_EPS_ADAM = 1e-6

HAS_TRITON = torch.cuda.is_available()

_BACKEND = "auto"          # 'auto' | 'triton' | 'eager'
_PRECISION = "tf32"        # 'tf32' | 'ieee'


def set_precision(name: str):
    global _PRECISION
    assert name in ("tf32", "ieee")
    _PRECISION = name


def set_backend(name: str):
    global _BACKEND
    assert name in ("auto", "triton", "eager")
    _BACKEND = name


def _precision_code(name: str) -> int:
    return _ops.GMDN_PREC_IEEE if name == "ieee" else _ops.GMDN_PREC_FAST


class _TritonScan:
    """Autograd entry with the reference's call signature (fast_scan.py:334)."""

    @staticmethod
    def apply(U, K, a, b, m, n, rule, ns):
        return _ops.state_scan(U, K, a, b, m, n, rule, ns, _precision_code(_PRECISION))


def fast_state_scan(U, K, a, b, m, n, rule: int, ns: int) -> torch.Tensor:
    """Pre-update state stack (B, H, N, dh, dh) from the B200 kernels."""
    if _BACKEND == "eager":
        raise RuntimeError("set_backend('eager'): the B200 build ships no eager scan; "
                           "use the reference module for the eager recurrence")
    if not U.is_cuda:
        raise RuntimeError("fast_state_scan: CUDA tensors required (no CPU fallback)")
    return _TritonScan.apply(U, K, a, b, m, n, rule, ns)


def __getattr__(name):
    if name in ("scan_eager", "manual_backward", "_msign_sq", "_msign_vjp", "_ns_step"):
        raise AttributeError(
            f"fast_scan.{name} is the reference's eager PyTorch code and is not part of the "
            "B200 build; import it from the reference module (see patch_reference)")
    raise AttributeError(name)
