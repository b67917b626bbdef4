"""kernrt_cuda_prepare_embedding_file: the token embedding taken from a
safetensors file and converted on the device by matrix_from_raw's rules
(hf.rs:151-191), checked bit for bit against the oracle's restatement of
those rules over the same payload, through the device embedding."""
import numpy as np
import pytest

import kernrt_b200
from tests import _data
from tests._parity import assert_bits_equal

pytestmark = pytest.mark.gpu

F32, BF16, Q8_0, Q8_0X4 = 0, 1, 2, 3
NAMES = {F32: "f32", BF16: "bf16", Q8_0: "q8_0", Q8_0X4: "q8_0x4"}


def payload(dtype, vocab, dim, seed):
    """A [vocab, dim] payload in the file's dtype, as raw bits (or f32)."""
    w = _data.lcg_normal(vocab * dim, seed, 0.0, 0.05).reshape(vocab, dim)
    if dtype == "F32":
        return w
    if dtype == "BF16":
        from oracle import oracle as o
        return o.f32_to_bf16_bits(w).reshape(vocab, dim)
    h = w.astype(np.float16).view(np.uint16).copy()
    # halves the widening must get right: zeros, subnormals, the extremes
    special = np.array([0x0000, 0x8000, 0x0001, 0x83FF, 0x0400, 0x7BFF, 0xFBFF, 0x3C00], np.uint16)
    h.ravel()[:special.size] = special
    return h


def expected_storage(dtype, storage, vocab, dim):
    aligned_q8 = dim % 32 == 0
    aligned_q8x4 = aligned_q8 and vocab % 4 == 0
    if dtype == "BF16" and storage == BF16:
        return "bf16"
    if dtype == "BF16" and storage == Q8_0 and aligned_q8:
        return "q8_0"
    if dtype == "BF16" and storage == Q8_0X4 and aligned_q8x4:
        return "q8_0x4"
    if storage == F32:
        return "f32"
    if storage == Q8_0X4 and aligned_q8x4:
        return "q8_0x4"
    return "bf16"


def embed_all(gpu, vocab, dim):
    toks = np.arange(vocab, dtype=np.int32)
    out = gpu.alloc(vocab * dim)
    for r, t in enumerate(toks):
        gpu.embed(int(t), out, r * dim)
    return toks, gpu.read(out, vocab * dim).reshape(vocab, dim)


@pytest.mark.parametrize("vocab,dim", [(100, 64), (101, 64), (24, 40)])
@pytest.mark.parametrize("storage", [F32, BF16, Q8_0, Q8_0X4])
@pytest.mark.parametrize("dtype", ["F32", "BF16", "F16"])
def test_embedding_from_file_follows_matrix_from_raw(gpu, oracle, tmp_path, dtype, storage, vocab, dim):
    raw = payload(dtype, vocab, dim, 700 + vocab + dim)
    # other tensors and metadata around the one that is read
    img = _data.safetensors_bytes([
        ("model.norm.weight", "F32", [dim], np.ones(dim, np.float32).tobytes()),
        ("model.embed_tokens.weight", dtype, [vocab, dim], np.ascontiguousarray(raw).tobytes()),
        ("lm_head.weight", "BF16", [2, dim], bytes(4 * dim)),
    ], metadata={"format": "pt"})
    path = tmp_path / "model.safetensors"
    path.write_bytes(img)
    gpu.prepare_embedding_file(str(path), "model.embed_tokens.weight", storage)
    assert gpu.storage() == expected_storage(dtype, storage, vocab, dim)
    kind, data, scales = oracle.table_from_raw(dtype, raw, storage)
    toks, got = embed_all(gpu, vocab, dim)
    assert_bits_equal(got, oracle.embed_rows(kind, data, scales, vocab, dim, toks), f"{dtype}->{NAMES[storage]}")


def test_f16_nan_and_inf_keep_their_bits(gpu, oracle, tmp_path):
    vocab, dim = 4, 8
    h = np.array([0x7C00, 0xFC00, 0x7C01, 0xFE00, 0x7E00, 0x3555, 0x0000, 0x8001] * 4, np.uint16).reshape(vocab, dim)
    path = tmp_path / "h.safetensors"
    path.write_bytes(_data.safetensors_bytes([("e", "F16", [vocab, dim], h.tobytes())]))
    gpu.prepare_embedding_file(str(path), "e", F32)
    _, got = embed_all(gpu, vocab, dim)
    assert got.view(np.uint32).tolist() == oracle.st_f16_to_f32(h).view(np.uint32).tolist()


def test_file_errors_leave_the_previous_table(gpu, oracle, tmp_path):
    vocab, dim = 8, 32
    table = _data.bf16_table(vocab, dim, 9)
    gpu.prepare_embedding(oracle.BF16, table, None, vocab, dim)
    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(_data.safetensors_bytes([("t3", "F32", [2, 2, 2], bytes(32))]))
    with pytest.raises(kernrt_b200.KernrtCudaError, match="weight file is missing"):
        gpu.prepare_embedding_file(str(bad), "model.embed_tokens.weight", BF16)
    with pytest.raises(kernrt_b200.KernrtCudaError, match="a weight matrix was not rank 2"):
        gpu.prepare_embedding_file(str(bad), "t3", BF16)
    with pytest.raises(kernrt_b200.KernrtCudaError, match="i/o error"):
        gpu.prepare_embedding_file(str(tmp_path / "absent.safetensors"), "t3", BF16)
    with pytest.raises(kernrt_b200.KernrtCudaError, match="unknown storage kind"):
        gpu.prepare_embedding_file(str(bad), "t3", 9)
    assert gpu.storage() == "bf16"
    toks, got = embed_all(gpu, vocab, dim)
    assert_bits_equal(got, oracle.embed_rows(oracle.BF16, table, None, vocab, dim, toks), "kept table")


def test_bf16_table_of_the_headline_size_streams_unchanged(gpu, oracle, tmp_path):
    """The SmolLM2-1.7B table (49 152 x 2048 bf16, 201 MB) through the chunked
    file reader: rows at the chunk boundaries and a seeded sample equal the
    file's bits."""
    vocab, dim = 49152, 2048
    table = _data.bf16_table_fast(vocab, dim, 11)
    path = tmp_path / "big.safetensors"
    path.write_bytes(_data.safetensors_bytes([("model.embed_tokens.weight", "BF16", [vocab, dim], table.tobytes())]))
    gpu.prepare_embedding_file(str(path), "model.embed_tokens.weight", BF16)
    assert gpu.storage() == "bf16"
    chunk_rows = (64 << 20) // (2 * dim)
    toks = np.unique(np.concatenate([np.arange(0, vocab, chunk_rows), np.arange(chunk_rows - 1, vocab, chunk_rows),
                                     _data.tokens(200, vocab, 12), [vocab - 1]])).astype(np.int32)
    out = gpu.alloc(toks.size * dim)
    for r, t in enumerate(toks):
        gpu.embed(int(t), out, r * dim)
    got = gpu.read(out, toks.size * dim).reshape(toks.size, dim)
    assert_bits_equal(got, oracle.bf16_to_f32(table[toks]), "201 MB bf16 table")
