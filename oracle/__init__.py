"""CPU oracle for the chunkwise gated fast-weight state scan.

TEST INFRASTRUCTURE ONLY. Nothing in the shipped package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker or as the timed CPU baseline.

Parity status: pinned. ``tests/golden/make_golden.py`` imports the reference
(``fast_scan.py`` and ``train_ablation.py``) in the development container and
records its outputs on seeded inputs; ``tests/test_oracle_golden.py`` checks
this restatement against those fixtures.
"""

from .scan_oracle import (NS_COEF, EPS_NORM, EPS_ADAM, msign_square,
                          msign_square_vjp, scan_forward, scan_forward_all,
                          scan_backward)
from .mixer_oracle import chunk_gate_scalars, token_weights, mixer_core_forward
from .epilogue_oracle import head_rmsnorm
from .prologue_oracle import mixer_prologue

__all__ = [
    "NS_COEF", "EPS_NORM", "EPS_ADAM", "msign_square", "msign_square_vjp",
    "scan_forward", "scan_forward_all", "scan_backward",
    "chunk_gate_scalars", "token_weights", "mixer_core_forward", "head_rmsnorm",
    "mixer_prologue",
]
