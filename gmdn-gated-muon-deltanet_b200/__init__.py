"""B200-native chunkwise gated fast-weight state scan (delta / muon / adam).

Public API
  state_scan(U, K, a, b, m, n, rule, ns, precision)     fast_scan.py:403 equivalent
  chunk_fast_weight(q, k, v, alpha, beta, mu, nu, rule, ns, chunk, precision)
                                                        train_ablation.py:142-187
  fast_scan                                             drop-in module for `fast_scan`
  patch_reference / patch_mixer                         hooks into the reference's modules

Importing the package loads ``libgmdn_b200.so`` (built by ``build.py``) and
raises if it is missing: there is no fallback implementation.
"""

from ._lib import GMDN_PREC_FAST, GMDN_PREC_IEEE, LIB_PATH, kernel_launches  # noqa: F401
from .ops import (ScanFunction, chunk_fast_weight, head_rmsnorm, mixer_prologue,  # noqa: F401
                  state_scan)
from .integration import patch_mixer, patch_reference  # noqa: F401
from . import fast_scan, sharding, workloads  # noqa: F401

__all__ = ["state_scan", "chunk_fast_weight", "head_rmsnorm", "mixer_prologue", "ScanFunction", "fast_scan", "workloads",
           "sharding", "patch_reference", "patch_mixer", "GMDN_PREC_IEEE", "GMDN_PREC_FAST",
           "kernel_launches", "LIB_PATH"]
