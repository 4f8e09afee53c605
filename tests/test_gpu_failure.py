"""Failure detection on the GPU without a fault: a bounded wait that runs out.

The kernels' every mbarrier wait gives up after a time limit, records the
give-up in a device status word, lets the CTA's other warps leave and returns.
``gmdn_selftest_wait_timeout`` runs that same wait on an mbarrier nothing
arrives on, with a short limit; the tests check the status word and that the
context still runs an ordinary op afterwards, and that the status read-back
of the chunk entry points reports a set word as GMDN_ERR_DEVICE.
"""

import ctypes
import time

import pytest
import torch

from conftest import load_pkg
from parity import TOL_BF16

GMDN_ERR_DEVICE = 5


@pytest.mark.gpu
def test_bounded_wait_gives_up_and_context_survives():
    pkg = load_pkg()
    lib = pkg._lib.lib
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = lib.gmdn_selftest_wait_timeout(ctypes.c_void_p(status.data_ptr()), 20_000_000,
                                        ctypes.c_void_p(stream.cuda_stream))
    assert rc == 0, lib.gmdn_last_error_string()
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    # bit 0: the wait gave up; bit 31 would mean it completed, which it cannot
    assert status.item() == 1
    assert 0.015 < waited < 5.0, waited
    # the context is intact: an ordinary mixer-core call still matches the oracle
    from test_gpu_chunk import compare
    inp = pkg.workloads.mixer_inputs(1, 2, 256, 128, rule=0, seed=90)
    compare(pkg, inp, 0, 3, 64, pkg.GMDN_PREC_FAST, torch.bfloat16, TOL_BF16)


@pytest.mark.gpu
def test_status_read_back_reports_a_give_up():
    pkg = load_pkg()
    lib = pkg._lib.lib
    word = torch.zeros(64, dtype=torch.int32, device="cuda")   # stands for a workspace
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.gmdn_chunk_status(ctypes.c_void_p(word.data_ptr()), stream) == 0
    rc = lib.gmdn_selftest_wait_timeout(ctypes.c_void_p(word.data_ptr()), 1_000_000, stream)
    assert rc == 0
    assert lib.gmdn_chunk_status(ctypes.c_void_p(word.data_ptr()), stream) == GMDN_ERR_DEVICE
    assert b"wait timed out" in lib.gmdn_last_error_string()
