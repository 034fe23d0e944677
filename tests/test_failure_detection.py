"""Failure detection without faulting a GPU.

* Host side (no GPU, no NCCL): ns_comm_selftest runs the communicator's own
  poll-with-deadline loop (the one behind non-blocking NCCL creation, the
  enqueue of collectives and the end-of-step wait) against a fake NCCL whose
  behaviour each scenario sets: work that finishes, work that never
  finishes, a peer's asynchronous error, a creation that never completes.
  The loop must return the right status within its deadline and abort the
  communicator exactly when it gives up.
* Device side (GPU): ns_selftest_device_wait launches a warp that waits, with
  the tcgen05 kernels' bounded wait routine, on an mbarrier nothing arrives
  at; the wait runs out after a short limit, the kernel returns, the next
  ns_kernel_health() reports NS_ERR_TIMEOUT once, and the context keeps
  working (a GEMM right after it is checked against the oracle).
"""
import time

import numpy as np
import pytest

from neuralsuite_b200 import _lib

NS_OK, NS_ERR_COMM, NS_ERR_TIMEOUT = _lib.NS_OK, _lib.NS_ERR_COMM, _lib.NS_ERR_TIMEOUT


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def selftest(lib, scenario, timeout_s):
    import ctypes

    aborts = ctypes.c_int(-1)
    t0 = time.perf_counter()
    rc = lib.ns_comm_selftest(scenario, timeout_s, ctypes.byref(aborts))
    return rc, aborts.value, time.perf_counter() - t0


def test_wait_that_finishes_returns_ok_without_abort(lib):
    rc, aborts, dt = selftest(lib, 0, 5.0)
    assert rc == NS_OK and aborts == 0
    assert dt < 1.0


def test_wait_that_never_finishes_times_out_and_aborts(lib):
    rc, aborts, dt = selftest(lib, 1, 0.2)
    assert rc == NS_ERR_TIMEOUT, lib.ns_last_error()
    assert b"deadline" in lib.ns_last_error()
    assert aborts == 1
    assert 0.2 <= dt < 5.0


def test_peer_error_aborts_before_the_deadline(lib):
    rc, aborts, dt = selftest(lib, 2, 30.0)
    assert rc == NS_ERR_COMM, lib.ns_last_error()
    assert b"remote error" in lib.ns_last_error()
    assert aborts == 1
    assert dt < 5.0  # the error, not the 30 s deadline, ended the wait


def test_nonblocking_creation_that_never_completes_times_out(lib):
    rc, aborts, dt = selftest(lib, 3, 0.2)
    assert rc == NS_ERR_TIMEOUT, lib.ns_last_error()
    assert b"creation" in lib.ns_last_error()
    assert aborts == 1


def test_nonblocking_creation_that_completes(lib):
    rc, aborts, _ = selftest(lib, 4, 5.0)
    assert rc == NS_OK and aborts == 0


def test_selftest_rejects_unknown_scenarios(lib):
    rc, _, _ = selftest(lib, 9, 1.0)
    assert rc == _lib.NS_ERR_INVALID_ARGUMENT


@pytest.mark.gpu
def test_device_wait_that_runs_out_reports_timeout_and_context_survives(cuda, port):
    import torch

    from neuralsuite_b200 import kernels as nk
    from tests._util import assert_close, normal, rng

    lib = _lib.load()
    nk.kernel_health()  # start from a clear flag
    t0 = time.perf_counter()
    _lib.check(lib.ns_selftest_device_wait(20000, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 10.0
    assert lib.ns_kernel_health() == NS_ERR_TIMEOUT
    assert b"bounded wait" in lib.ns_last_error()
    assert lib.ns_kernel_health() == NS_OK  # reported once, then cleared
    r = rng(77)
    A, B = normal(r, (256, 128)), normal(r, (128, 192))
    C = nk.gemm(torch.as_tensor(A, device=cuda), torch.as_tensor(B, device=cuda))
    torch.cuda.synchronize()
    assert_close(C.cpu().numpy(), port.matmul(A, B), A.astype(np.float64) @ B, what="gemm after")
    nk.kernel_health()
