"""gmdn_scan_fwd_noalloc (static device scratch) against gmdn_scan_fwd.

The allocation-free entry point runs the same exact-fp32 forward as
gmdn_scan_fwd with its scratch in a fixed device array of the library.  Two
calls in a row (muon, then adam on other inputs) check that what the first call
leaves in the shared array does not reach the second call's result; each is
compared with gmdn_scan_fwd given a fresh workspace, within the fp32 tolerance
the other scan tests use.  The file is named to be collected last, and passes
both alone and after the rest of the suite.
"""
import ctypes

import pytest
import torch

from conftest import load_pkg
from parity import TOL_FP32, rel

pytestmark = pytest.mark.gpu

B, H, N, DH, NS = 2, 3, 6, 64, 3


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _inputs(seed):
    pkg = load_pkg()
    return [t.cuda().contiguous() for t in pkg.workloads.scan_inputs(B, H, N, DH, seed=seed)]


def _saved(lib, rule):
    nbytes = max(lib.gmdn_scan_saved_bytes(B, H, N, DH, rule), 1)
    return torch.zeros(nbytes, dtype=torch.uint8, device="cuda")


def _fwd_workspace(lib, ins, rule):
    S = torch.empty_like(ins[0])
    saved = _saved(lib, rule)
    wsz = lib.gmdn_scan_workspace_bytes(B, H, N, DH, rule, NS, 0)
    ws = torch.empty(wsz, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.gmdn_scan_fwd(*[_ptr(t) for t in ins], _ptr(S), _ptr(saved), _ptr(ws), wsz,
                           B, H, N, DH, rule, NS, 0, stream)
    assert rc == 0, lib.gmdn_last_error_string().decode()
    return S, saved


def _fwd_noalloc(lib, ins, rule):
    S = torch.full_like(ins[0], float("nan"))
    saved = _saved(lib, rule)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.gmdn_scan_fwd_noalloc(*[_ptr(t) for t in ins], _ptr(S), _ptr(saved),
                                   B, H, N, DH, rule, NS, 0, stream)
    assert rc == 0, lib.gmdn_last_error_string().decode()
    return S, saved


def test_noalloc_scan_fwd_matches_workspace_entry_point():
    lib = load_pkg()._lib.lib
    for call, (rule, seed) in enumerate([(1, 11), (2, 12)]):
        ins = _inputs(seed)
        S_ref, saved_ref = _fwd_workspace(lib, ins, rule)
        S, saved = _fwd_noalloc(lib, ins, rule)
        torch.cuda.synchronize()
        assert torch.isfinite(S).all(), f"call {call}: non-finite states"
        err = rel(S.cpu(), S_ref.cpu())
        assert err <= TOL_FP32, f"call {call} (rule {rule}): states rel err {err:.3e}"
        # `saved` holds the pre-update moment histories (fp32) for muon / adam
        m = saved.view(torch.float32).cpu()
        m_ref = saved_ref.view(torch.float32).cpu()
        err = rel(m, m_ref)
        assert err <= TOL_FP32, f"call {call} (rule {rule}): moment history rel err {err:.3e}"


def test_noalloc_scan_fwd_rejects_sizes_beyond_its_scratch():
    lib = load_pkg()._lib.lib
    x = torch.zeros(16, device="cuda")
    # 43 (b,h) pairs at dh 128 need 43 * 6 * 128 * 128 * 4 bytes > 16 MiB
    rc = lib.gmdn_scan_fwd_noalloc(*[_ptr(x)] * 8, 1, 43, 1, 128, 0, 3, 0,
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 3
    assert b"static scratch" in lib.gmdn_last_error_string()
