"""ctypes binding of ``libgmdn_b200.so`` (the C ABI in include/gmdn_scan.h).

The library is built in-tree by ``build.py``.  There is no fallback: if the
shared library is missing or cannot be loaded, importing this module raises.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgmdn_b200.so")

GMDN_PREC_IEEE = 0
GMDN_PREC_FAST = 1

ERR_NAMES = {1: "invalid argument", 2: "unsupported", 3: "workspace too small",
             4: "CUDA error", 5: "device-side failure"}


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with "
            f"`python {os.path.join(_HERE, 'build.py')}` (needs nvcc, targets sm_100a)")
    return ctypes.CDLL(LIB_PATH)


lib = _load()

_p = ctypes.c_void_p
_i = ctypes.c_int
_z = ctypes.c_size_t

lib.gmdn_abi_version.restype = _i
lib.gmdn_abi_version.argtypes = []
lib.gmdn_last_error_string.restype = ctypes.c_char_p
lib.gmdn_last_error_string.argtypes = []
lib.gmdn_kernel_launches.restype = ctypes.c_uint64
lib.gmdn_kernel_launches.argtypes = []
lib.gmdn_chunk_bwd_fused_tiles.restype = _i
lib.gmdn_chunk_bwd_fused_tiles.argtypes = [_i] * 8
lib.gmdn_selftest_wait_timeout.restype = _i
lib.gmdn_selftest_wait_timeout.argtypes = [_p, ctypes.c_uint64, _p]
lib.gmdn_prof_enable.restype = None
lib.gmdn_prof_enable.argtypes = [_i]
lib.gmdn_prof_report.restype = ctypes.c_char_p
lib.gmdn_prof_report.argtypes = []

lib.gmdn_scan_saved_bytes.restype = _z
lib.gmdn_scan_saved_bytes.argtypes = [_i] * 5
lib.gmdn_scan_workspace_bytes.restype = _z
lib.gmdn_scan_workspace_bytes.argtypes = [_i] * 7
lib.gmdn_scan_fwd.restype = _i
lib.gmdn_scan_fwd.argtypes = [_p] * 9 + [_z] + [_i] * 7 + [_p]
lib.gmdn_scan_fwd_noalloc.restype = _i
lib.gmdn_scan_fwd_noalloc.argtypes = [_p] * 8 + [_i] * 7 + [_p]
lib.gmdn_scan_bwd.restype = _i
lib.gmdn_scan_bwd.argtypes = [_p] * 16 + [_z] + [_i] * 7 + [_p]

lib.gmdn_chunk_saved_bytes.restype = _z
lib.gmdn_chunk_saved_bytes.argtypes = [_i] * 8
lib.gmdn_chunk_workspace_bytes.restype = _z
lib.gmdn_chunk_workspace_bytes.argtypes = [_i] * 8
lib.gmdn_chunk_fwd.restype = _i
lib.gmdn_chunk_fwd.argtypes = [_p] * 10 + [_z] + [_i] * 8 + [_p]
lib.gmdn_chunk_bwd.restype = _i
lib.gmdn_chunk_bwd.argtypes = [_p] * 17 + [_z] + [_i] * 8 + [_p]
lib.gmdn_chunk_saved_bytes_ex.restype = _z
lib.gmdn_chunk_saved_bytes_ex.argtypes = [_i] * 9
lib.gmdn_chunk_workspace_bytes_ex.restype = _z
lib.gmdn_chunk_workspace_bytes_ex.argtypes = [_i] * 9
lib.gmdn_chunk_status.restype = _i
lib.gmdn_chunk_status.argtypes = [_p, _p]
lib.gmdn_chunk_fwd_ex.restype = _i
lib.gmdn_chunk_fwd_ex.argtypes = [_p] * 10 + [_z] + [_i] * 9 + [_p]
lib.gmdn_chunk_bwd_ex.restype = _i
lib.gmdn_chunk_bwd_ex.argtypes = [_p] * 17 + [_z] + [_i] * 9 + [_p]

lib.gmdn_mixer_prologue_fwd.restype = _i
lib.gmdn_mixer_prologue_fwd.argtypes = [_p] * 8 + [_i] * 6 + [_p]
lib.gmdn_mixer_prologue_bwd.restype = _i
lib.gmdn_mixer_prologue_bwd.argtypes = [_p] * 12 + [_i] * 6 + [_p]
lib.gmdn_head_rmsnorm_fwd.restype = _i
lib.gmdn_head_rmsnorm_fwd.argtypes = [_p] * 3 + [_i] * 4 + [ctypes.c_float] + [_i] * 2 + [_p]
lib.gmdn_head_rmsnorm_bwd.restype = _i
lib.gmdn_head_rmsnorm_bwd.argtypes = [_p] * 5 + [_i] * 4 + [ctypes.c_float] + [_i] * 2 + [_p]


def check(rc: int, what: str) -> None:
    """Raise RuntimeError carrying the library's message when rc != 0."""
    if rc != 0:
        msg = lib.gmdn_last_error_string().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({ERR_NAMES.get(rc, rc)}): {msg}")


def kernel_launches() -> int:
    return int(lib.gmdn_kernel_launches())


def chunk_bwd_fused_tiles(B: int, H: int, T: int, dh: int, chunk: int, rule: int,
                          precision: int, io_f32: bool = False) -> int:
    """Tiles (chunk-heads) whose token gradients the fused delta backward
    computes beside its reverse chains; 0 where the backward is the two plain
    launches."""
    return int(lib.gmdn_chunk_bwd_fused_tiles(B, H, T, dh, chunk, rule, precision, int(io_f32)))


def prof_enable(on: bool) -> None:
    """Bracket every kernel launch with CUDA events on its own stream."""
    lib.gmdn_prof_enable(1 if on else 0)


def prof_report() -> dict:
    """{kernel name: (total ms, launches)} since the previous report; waits for
    the recorded events."""
    import json
    return {k: (v[0], v[1]) for k, v in json.loads(lib.gmdn_prof_report().decode()).items()}
