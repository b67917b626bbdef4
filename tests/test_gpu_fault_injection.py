"""Host-side fault injection: a device allocation that fails.

KERNRT_CUDA_FAIL_ALLOC=n (read once when a context is created; unset, nothing
is injected) makes that context's n-th buffer allocation fail as an exhausted
device would.  The call reports KERNRT_E_CUDA with cudaMalloc's message, the
way the reference reports a backend that cannot start (BackendError.detail,
src/backends/mod.rs:192-213), and the context keeps computing: the buffers it
already holds and the ones allocated afterwards give bit-exact results.  No
GPU fault is involved: the allocation is refused on the host.
"""
import os

import numpy as np
import pytest

import kernrt_b200
from tests import _data
from tests._parity import assert_bits_equal

pytestmark = pytest.mark.gpu


def test_failed_allocation_reports_and_the_context_keeps_computing(oracle):
    rows, dim, eps = 40, 256, 1e-5
    x = _data.lcg_normal(rows * dim, 801).reshape(rows, dim)
    w = (1 + 0.1 * _data.lcg_normal(dim, 802)).astype(np.float32)
    os.environ["KERNRT_CUDA_FAIL_ALLOC"] = "3"
    try:
        b = kernrt_b200.CudaBackend(0)
    finally:
        del os.environ["KERNRT_CUDA_FAIL_ALLOC"]
    with b:
        hx, hw = b.upload(x), b.upload(w)  # allocations 1 and 2
        with pytest.raises(kernrt_b200.KernrtCudaError) as e:
            b.alloc(rows * dim)  # allocation 3 is refused
        assert e.value.code == kernrt_b200.E_CUDA
        assert "cudaMalloc" in str(e.value) and "memory" in str(e.value)
        out = b.alloc(rows * dim)  # allocation 4 succeeds
        b.rms_norm(out, hx, hw, rows, dim, eps)
        assert_bits_equal(b.read(out, rows * dim).reshape(rows, dim), oracle.rms_norm(x, w, eps),
                          "rms_norm after a refused allocation")
    with kernrt_b200.CudaBackend(0) as b2:  # a new context injects nothing
        handles = [b2.alloc(16) for _ in range(5)]
        assert len(set(handles)) == 5
