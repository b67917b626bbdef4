"""kernrt_cuda_embed_rows_noalloc against the regular embed path, through the C ABI.

Callers such as a host runtime that owns all device memory through its own
pool, or a serving loop that must not trigger the device-wide synchronisation
of cudaMalloc/cudaFree, cannot let the library allocate.  The no-allocation
gather serves them from a fixed scratch array compiled into the library.  This
test checks that it returns exactly what kernrt_cuda_embed returns, on two
calls in a row (the scratch keeps the previous call's contents), and that it
rejects a row count above its fixed limit.  All device memory the test uses is
allocated by the test itself, before the calls.

The file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""
import numpy as np
import pytest

import kernrt_b200
from tests import _data
from tests._parity import assert_bits_equal

pytestmark = pytest.mark.gpu


def _embed_reference_path(b, tokens, dim):
    out = b.alloc(len(tokens) * dim)
    for r, t in enumerate(tokens):
        b.embed(int(t), out, r * dim)
    return b.read(out, len(tokens) * dim)


@pytest.mark.parametrize("kind,vocab,dim", [(kernrt_b200.BF16, 3000, 2048), (kernrt_b200.Q8_0, 2000, 1024),
                                            (kernrt_b200.F32, 500, 36)])
def test_noalloc_gather_matches_embed_on_two_calls(kind, vocab, dim):
    with kernrt_b200.CudaBackend(0) as b:
        scales = None
        if kind == kernrt_b200.BF16:
            table = _data.bf16_table_fast(vocab, dim, 11)
        elif kind == kernrt_b200.Q8_0:
            table, scales = _data.q8_table_fast(vocab, dim, 12)
        else:
            table = np.random.default_rng(13).standard_normal((vocab, dim), dtype=np.float32)
        b.prepare_embedding(kind, table, scales, vocab, dim)
        dev_table = b.upload_bytes(table)
        dev_scales = b.upload_bytes(scales) if scales is not None else 0
        outs = [b.alloc(n * dim) for n in (1500, 777)]
        for call, (n, out) in enumerate(zip((1500, 777), outs)):
            tokens = _data.tokens(n, vocab, 100 + call)
            want = _embed_reference_path(b, tokens, dim)
            kernrt_b200.embed_rows_noalloc(0, kind, b.device_ptr(dev_table),
                                           b.device_ptr(dev_scales) if dev_scales else 0, vocab, dim,
                                           tokens, b.device_ptr(out), b.stream())
            got = b.read(out, n * dim)  # the backend's stream carried the call
            assert_bits_equal(got, want, f"no-alloc gather, call {call + 1}")


def test_noalloc_gather_scalar_path_default_stream_and_device():
    """An output one float past a 16-byte boundary and a bf16 width of 40 take
    the gather's element-wise form; the call goes on the legacy default stream
    (stream 0) and leaves the caller's current device as it found it."""
    import torch

    vocab, dim, n = 700, 40, 333
    with kernrt_b200.CudaBackend(0) as b:
        table = _data.bf16_table_fast(vocab, dim, 15)
        b.prepare_embedding(kernrt_b200.BF16, table, None, vocab, dim)
        dev_table = b.upload_bytes(table)
        out = b.alloc(n * dim + 4)
        for call in range(2):
            tokens = _data.tokens(n, vocab, 300 + call)
            want = _embed_reference_path(b, tokens, dim)
            before = torch.cuda.current_device()
            kernrt_b200.embed_rows_noalloc(0, kernrt_b200.BF16, b.device_ptr(dev_table), 0, vocab, dim, tokens,
                                           b.device_ptr(out) + 4, 0)
            assert torch.cuda.current_device() == before
            torch.cuda.synchronize()
            got = b.read_bytes(out, (n * dim + 1) * 4, np.float32)[1:]
            assert_bits_equal(got, want, f"no-alloc gather, unaligned rows, call {call + 1}")


def test_noalloc_gather_rejects_what_it_cannot_hold():
    with kernrt_b200.CudaBackend(0) as b:
        vocab, dim = 64, 128
        table = _data.bf16_table_fast(vocab, dim, 14)
        dev_table = b.upload_bytes(table)
        out = b.alloc(16 * dim)
        too_many = np.zeros(kernrt_b200.NOALLOC_MAX_ROWS + 1, np.int32)
        with pytest.raises(kernrt_b200.KernrtCudaError) as e:
            kernrt_b200.embed_rows_noalloc(0, kernrt_b200.BF16, b.device_ptr(dev_table), 0, vocab, dim,
                                           too_many, b.device_ptr(out), b.stream())
        assert e.value.code == kernrt_b200.E_INVALID
        assert "exceed" in str(e.value)
        with pytest.raises(kernrt_b200.KernrtCudaError) as e:
            kernrt_b200.embed_rows_noalloc(0, kernrt_b200.BF16, b.device_ptr(dev_table), 0, vocab, dim,
                                           np.array([3, vocab], np.int32), b.device_ptr(out), b.stream())
        assert e.value.code == kernrt_b200.E_INVALID
        # still usable after a rejected call
        tokens = np.array([5, 0, 63], np.int32)
        kernrt_b200.embed_rows_noalloc(0, kernrt_b200.BF16, b.device_ptr(dev_table), 0, vocab, dim, tokens,
                                       b.device_ptr(out), b.stream())
        got = b.read(out, 3 * dim)
        want = (table[tokens].astype(np.uint32) << 16).view(np.float32).ravel()
        assert_bits_equal(got, want, "after rejection")
