"""Comparison helpers for the GPU parity tests.

Bit parity compares raw IEEE bit patterns (so -0.0 vs +0.0 and NaN payloads
count).  SwiGLU, the one op that calls CUDA's expf instead of glibc's, is held
to the stated tolerance: per element |g - r| <= 1e-5 * |r| (for r != 0) and
g == 0 where r == 0.
"""
import numpy as np

SILU_RTOL = 1e-5


def assert_bits_equal(got, want, what=""):
    got = np.ascontiguousarray(got)
    want = np.ascontiguousarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} vs {want.shape}"
    if got.dtype == np.float32:
        g, w = got.view(np.uint32), want.view(np.uint32)
    else:
        g, w = got, want
    bad = np.flatnonzero(g.ravel() != w.ravel())
    if bad.size:
        i = bad[0]
        raise AssertionError(
            f"{what}: {bad.size} of {g.size} elements differ; first at {i}: "
            f"got {got.ravel()[i]!r} want {want.ravel()[i]!r}")


def assert_close_rel(got, want, rtol=SILU_RTOL, what=""):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    assert got.shape == want.shape
    zero = want == 0
    assert np.all(got[zero] == 0), f"{what}: nonzero where the oracle is zero"
    nz = ~zero
    rel = np.abs(got[nz] - want[nz]) / np.abs(want[nz])
    worst = float(rel.max()) if rel.size else 0.0
    assert worst <= rtol, f"{what}: max relative error {worst:.3e} > {rtol:.0e}"
    return worst
