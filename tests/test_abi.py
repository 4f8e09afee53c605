"""CPU checks of the C ABI: the library loads, exports every declared symbol,
and rejects bad arguments before touching a device."""
import ctypes
import os
import re

import pytest
import torch

from conftest import ROOT, load_pkg

HEADER = os.path.join(ROOT, "include", "gmdn_scan.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gmdn_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    pkg = load_pkg()
    lib = ctypes.CDLL(pkg.LIB_PATH)
    names = declared_functions()
    assert len(names) >= 12
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version_and_sizes():
    from importlib import import_module
    lib = import_module("gmdn-gated-muon-deltanet_b200._lib").lib
    assert lib.gmdn_abi_version() == 1
    # config-1 shape: B8 H16 N64 dh128
    per = 8 * 16 * 64 * 128 * 128 * 4
    assert lib.gmdn_scan_saved_bytes(8, 16, 64, 128, 0) == 0
    assert lib.gmdn_scan_saved_bytes(8, 16, 64, 128, 1) >= per
    assert lib.gmdn_scan_saved_bytes(8, 16, 64, 128, 2) >= 2 * per
    assert lib.gmdn_scan_workspace_bytes(8, 16, 64, 128, 1, 5, 0) > 0
    assert lib.gmdn_chunk_saved_bytes(8, 16, 4096, 128, 64, 0, 5, 0) >= per
    assert lib.gmdn_chunk_workspace_bytes(8, 16, 4096, 128, 64, 0, 5, 0) > 0
    assert lib.gmdn_scan_saved_bytes(8, 16, 64, 100, 0) == 0  # unsupported dh


@pytest.mark.parametrize("bad", [
    dict(rule=3), dict(rule=-1), dict(ns=-1), dict(dh=48), dict(precision=7), dict(B=-2),
])
def test_scan_fwd_rejects_bad_arguments(bad):
    from importlib import import_module
    L = import_module("gmdn-gated-muon-deltanet_b200._lib")
    args = dict(B=1, H=1, N=2, dh=16, rule=0, ns=3, precision=0)
    args.update(bad)
    null = ctypes.c_void_p(None)
    rc = L.lib.gmdn_scan_fwd(*([null] * 9), 0, args["B"], args["H"], args["N"], args["dh"],
                             args["rule"], args["ns"], args["precision"], null)
    assert rc in (1, 2)
    assert L.lib.gmdn_last_error_string().decode()


def test_scan_fwd_rejects_null_pointers_and_small_workspace():
    from importlib import import_module
    L = import_module("gmdn-gated-muon-deltanet_b200._lib")
    null = ctypes.c_void_p(None)
    rc = L.lib.gmdn_scan_fwd(*([null] * 9), 0, 1, 1, 2, 16, 0, 3, 0, null)
    assert rc == 1 and "null" in L.lib.gmdn_last_error_string().decode()
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: the size check fails first
    rc = L.lib.gmdn_scan_fwd(*([fake] * 9), 16, 1, 1, 2, 16, 0, 3, 0, null)
    assert rc == 3 and "workspace" in L.lib.gmdn_last_error_string().decode()
    with pytest.raises(RuntimeError, match="workspace"):
        L.check(rc, "gmdn_scan_fwd")


def test_chunk_rejects_bad_chunk_and_seq_len():
    from importlib import import_module
    L = import_module("gmdn-gated-muon-deltanet_b200._lib")
    null = ctypes.c_void_p(None)
    rc = L.lib.gmdn_chunk_fwd(*([null] * 10), 0, 1, 1, 128, 64, 48, 0, 3, 0, null)
    assert rc == 2
    rc = L.lib.gmdn_chunk_fwd(*([null] * 10), 0, 1, 1, 100, 64, 64, 0, 3, 0, null)
    assert rc == 1 and "multiple" in L.lib.gmdn_last_error_string().decode()
    # empty input is a no-op
    assert L.lib.gmdn_chunk_fwd(*([null] * 10), 0, 0, 1, 128, 64, 64, 0, 3, 0, null) == 0


def test_ops_refuse_cpu_tensors():
    pkg = load_pkg()
    U = torch.zeros(1, 1, 2, 16, 16)
    g = torch.ones(1, 1, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.state_scan(U, U, g, g, g, g, 0, 3)
    q = torch.zeros(1, 1, 64, 16)
    gt = torch.ones(1, 1, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.chunk_fast_weight(q, q, q, gt, gt, gt, None, 0, 3, 64)


def test_ops_validate_shapes():
    pkg = load_pkg()
    U = torch.zeros(1, 1, 2, 16, 8)
    g = torch.ones(1, 1, 2)
    with pytest.raises(ValueError):
        pkg.state_scan(U, U, g, g, g, g, 0, 3)
    q = torch.zeros(1, 1, 100, 16)
    gt = torch.ones(1, 1, 100)
    with pytest.raises(ValueError, match="multiple"):
        pkg.chunk_fast_weight(q, q, q, gt, gt, gt, None, 0, 3, 64)
    q = torch.zeros(1, 1, 64, 16)
    gt = torch.ones(1, 1, 64)
    with pytest.raises(ValueError, match="nu"):
        pkg.chunk_fast_weight(q, q, q, gt, gt, gt, None, 2, 3, 64)


def test_fast_scan_shim_mirrors_reference_knobs():
    fs = load_pkg().fast_scan
    fs.set_backend("auto")
    fs.set_precision("ieee")
    with pytest.raises(AssertionError):
        fs.set_backend("cuda")
    with pytest.raises(AssertionError):
        fs.set_precision("bf16")
    U = torch.zeros(1, 1, 2, 16, 16)
    g = torch.ones(1, 1, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        fs.fast_state_scan(U, U, g, g, g, g, 0, 3)
    fs.set_backend("eager")
    with pytest.raises(RuntimeError, match="eager"):
        fs.fast_state_scan(U, U, g, g, g, g, 0, 3)
    fs.set_backend("auto")
    fs.set_precision("tf32")
    with pytest.raises(AttributeError, match="reference"):
        fs.scan_eager  # noqa: B018
    assert (fs.NS_A, fs.NS_B, fs.NS_C) == (3.4445, -4.7750, 2.0315)


def test_patch_reference_swaps_only_the_kernel_class():
    import types
    pkg = load_pkg()
    sentinel = object()
    mod = types.SimpleNamespace(_PRECISION="tf32", HAS_TRITON=False, _TritonScan=None,
                                scan_eager=sentinel)
    pkg.patch_reference(mod)
    assert mod.HAS_TRITON is True and mod.scan_eager is sentinel
    assert hasattr(mod._TritonScan, "apply")


def _aligned_addr():
    # a 16-byte aligned host address: the checks below return before any
    # device access, so the pointer is never dereferenced
    buf = (ctypes.c_char * 64)()
    return buf, ctypes.c_void_p((ctypes.addressof(buf) + 15) // 16 * 16)


def test_epilogue_and_prologue_reject_bad_arguments():
    from importlib import import_module
    lib = import_module("gmdn-gated-muon-deltanet_b200._lib").lib
    _keep, p = _aligned_addr()
    null = ctypes.c_void_p(None)
    stream = ctypes.c_void_p(None)
    # head_rmsnorm: unsupported dh, null pointer, misaligned pointer, negative size
    assert lib.gmdn_head_rmsnorm_fwd(p, p, p, 1, 2, 8, 48, -1.0, 1, 1, stream) == 2
    assert lib.gmdn_head_rmsnorm_fwd(p, null, p, 1, 2, 8, 64, -1.0, 1, 1, stream) == 1
    bad = ctypes.c_void_p(p.value + 2)
    assert lib.gmdn_head_rmsnorm_fwd(bad, p, p, 1, 2, 8, 64, -1.0, 1, 1, stream) == 1
    assert lib.gmdn_head_rmsnorm_bwd(p, p, null, p, p, 1, 2, 8, 64, -1.0, 1, 1, stream) == 1
    assert lib.gmdn_head_rmsnorm_fwd(p, p, p, -1, 2, 8, 64, -1.0, 1, 1, stream) == 1
    # mixer_prologue: bad n_gates, unsupported dh, null pointer, too large
    assert lib.gmdn_mixer_prologue_fwd(p, p, p, p, p, p, p, p, 1, 8, 2, 64, 5, 1, stream) == 1
    assert lib.gmdn_mixer_prologue_fwd(p, p, p, p, p, p, p, p, 1, 8, 2, 48, 3, 1, stream) == 2
    assert lib.gmdn_mixer_prologue_fwd(p, p, null, p, p, p, p, p, 1, 8, 2, 64, 3, 1, stream) == 1
    assert lib.gmdn_mixer_prologue_bwd(p, p, p, p, p, p, p, p, p, p, p, null, 1, 8, 2, 64, 3, 1,
                                       stream) == 1
    assert lib.gmdn_mixer_prologue_fwd(p, p, p, p, p, p, p, p, 4096, 65536, 16, 128, 3, 0,
                                       stream) == 2
    assert b"2^31" in lib.gmdn_last_error_string()


def test_epilogue_and_prologue_ops_validate_on_cpu():
    pkg = load_pkg()
    o = torch.zeros(1, 2, 8, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.head_rmsnorm(o, torch.ones(64))
    with pytest.raises(ValueError):
        pkg.head_rmsnorm(o, torch.ones(32))
    u = torch.zeros(1, 8, 3 * 2 * 64)
    gl = torch.zeros(1, 8, 3 * 2)
    w, b = torch.zeros(3 * 2 * 64, 1, 4), torch.zeros(3 * 2 * 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.mixer_prologue(u, w, b, gl, 2)
    with pytest.raises(ValueError):
        pkg.mixer_prologue(u, w, b, torch.zeros(1, 8, 5 * 2), 2)
    with pytest.raises(ValueError):
        pkg.mixer_prologue(u, torch.zeros(3 * 2 * 64, 1, 3), b, gl, 2)
