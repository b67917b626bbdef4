"""Every spin-wait in the kernels gives up after a cycle limit and reports
through the device error word instead of hanging the GPU.  The wait is run
out on purpose on an mbarrier phase that nothing completes (no copy in
flight, no fault): the call reports the timeout, and the context keeps
computing bit for bit afterwards."""
import numpy as np
import pytest

import kernrt_b200
from tests import _data
from tests._parity import assert_bits_equal

pytestmark = pytest.mark.gpu


def rms_norm_roundtrip(gpu, oracle, seed):
    rows, dim = 9, 256
    x = _data.lcg_normal(rows * dim, seed).reshape(rows, dim)
    w = _data.lcg_normal(dim, seed + 1, 1.0, 0.1)
    hx, hw, ho = gpu.upload(x), gpu.upload(w), gpu.alloc(rows * dim)
    gpu.rms_norm(ho, hx, hw, rows, dim, 1e-5)
    got = gpu.read(ho, rows * dim).reshape(rows, dim)
    assert_bits_equal(got, oracle.rms_norm(x, w, 1e-5), "rms_norm after a timeout")


def test_a_wait_that_runs_out_reports_and_the_context_survives(gpu, oracle):
    gpu.selftest_wait(1000, True)  # the phase completes: no error
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu.selftest_wait(2_000_000, False)  # ~1 ms of SM clock, then give up
    assert e.value.code == kernrt_b200.E_DEVICE
    assert "timed out" in str(e.value)
    rms_norm_roundtrip(gpu, oracle, 31)
    gpu.selftest_wait(1000, True)  # the error word was cleared
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu.selftest_wait(50_000, False)
    assert e.value.code == kernrt_b200.E_DEVICE
    rms_norm_roundtrip(gpu, oracle, 33)


def test_the_wait_limit_is_capped(gpu):
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu.selftest_wait(1 << 40, False)
    assert e.value.code == kernrt_b200.E_INVALID
