"""Failure detection on the GPU without a fault, a trap or a hang.

Every device-side wait in libg16 is bounded: on expiry the waiting role records G16_ERR_TIMEOUT in
the device status word and raises its CTA's abort flag, the other roles leave their own waits as
soon as they see the flag, and the kernel returns. g16_selftest_wait_timeout runs exactly that
machinery on an mbarrier that nothing arrives on, with a short limit, so these tests make a wait run
out and check that (1) the status word reports it, (2) the other role left early instead of waiting
out its own 1 s limit, (3) clearing the status works and (4) the context stays usable: a normal
GEMM afterwards is correct and leaves the status clean."""
import time

import pytest
import torch

import gtx16_fp16 as g
from gtx16_fp16 import _native

from _tol import assert_close_fp64

pytestmark = pytest.mark.gpu


def _run_selftest(limit_us):
    dev = torch.cuda.current_device()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _native.check(_native.lib().g16_selftest_wait_timeout(limit_us, _native.stream_handle(dev)),
                  "g16_selftest_wait_timeout")
    torch.cuda.synchronize()
    return time.perf_counter() - t0


def test_expired_wait_is_reported_and_unwinds(cuda_ok):
    assert _native.device_status(clear=True) in (_native.OK, _native.ERR_TIMEOUT)
    assert _native.device_status() == _native.OK
    dt = _run_selftest(2000)  # 2 ms on a barrier nothing arrives on
    assert _native.device_status() == _native.ERR_TIMEOUT
    # the second role (1 s limit) left on the abort flag, so the kernel ended long before 1 s
    assert dt < 0.5, f"kernel took {dt:.3f} s: the abort flag did not end the other wait"
    assert _native.device_status(clear=True) == _native.ERR_TIMEOUT
    assert _native.device_status() == _native.OK


def test_context_usable_after_a_timeout(cuda_ok):
    _run_selftest(1000)
    assert _native.device_status(clear=True) == _native.ERR_TIMEOUT
    torch.manual_seed(3)
    x = torch.randn(300, 1024, device="cuda")
    w = (torch.randn(1024, 768, device="cuda") * 0.03).half()
    b = torch.randn(768, device="cuda")
    y = g.mm_t(x, w, b, torch.float32)
    assert_close_fp64(y, x, w, b, torch.float32, "GEMM after a timeout")
    assert _native.device_status() == _native.OK


@pytest.mark.parametrize("limit_us", [1, 100, 20000])
def test_timeout_limits(cuda_ok, limit_us):
    dt = _run_selftest(limit_us)
    assert _native.device_status(clear=True) == _native.ERR_TIMEOUT
    assert dt >= limit_us * 1e-6 * 0.5  # the wait really waited (host clock, coarse)
    assert dt < 0.5
