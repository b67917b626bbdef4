"""The safetensors header reader behind kernrt_cuda_prepare_embedding_file
(host code, no GPU): src/formats/safetensors.rs's read_with checks and its
tests (:388-537), and the oracle's payload widening pinned to the reference's
known answers."""
import numpy as np
import pytest

import kernrt_b200
from tests import _data


@pytest.fixture
def st_file(tmp_path):
    def make(image: bytes, name="t.safetensors"):
        p = tmp_path / name
        p.write_bytes(image)
        return str(p)

    return make


def err(path, name="w"):
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        kernrt_b200.safetensors_tensor(path, name)
    assert e.value.code == kernrt_b200.E_INVALID
    return str(e.value)


def f32b(*v):
    return np.asarray(v, np.float32).tobytes()


def test_roundtrip_preserves_names_shapes_and_offsets(st_file):
    # safetensors.rs:415-426
    img = _data.safetensors_bytes([("fc1.weight", "F32", [2, 3], f32b(1, 2, 3, 4, 5, 6)),
                                   ("fc1.bias", "F32", [2], f32b(-1.5, 2.5))])
    p = st_file(img)
    w = kernrt_b200.safetensors_tensor(p, "fc1.weight")
    b = kernrt_b200.safetensors_tensor(p, "fc1.bias")
    assert (w["dtype"], w["shape"], w["bytes"]) == ("F32", (2, 3), 24)
    assert (b["dtype"], b["shape"], b["bytes"]) == ("F32", (2,), 8)
    assert np.array_equal(np.frombuffer(img[w["offset"]:w["offset"] + 24], np.float32), [1, 2, 3, 4, 5, 6])
    assert np.array_equal(np.frombuffer(img[b["offset"]:b["offset"] + 8], np.float32), [-1.5, 2.5])


def test_skips_the_metadata_entry(st_file):
    # safetensors.rs:428-441
    p = st_file(_data.safetensors_bytes([("w", "F32", [1], f32b(7.0))], metadata={"format": "pt"}))
    assert kernrt_b200.safetensors_tensor(p, "w")["shape"] == (1,)
    assert "missing" in err(p, "__metadata__")


def test_rejects_unsupported_dtype(st_file):
    # safetensors.rs:443-450
    p = st_file(_data.safetensors_bytes([("w", "I32", [1], f32b(0.0))]))
    assert err(p) == 'unsupported dtype "I32" (F32, BF16 and F16 are read)'


def test_reads_bf16_and_f16_entries(st_file):
    # safetensors.rs:471-485: the payloads of the reference's known answers
    p = st_file(_data.safetensors_bytes([("b", "BF16", [3], bytes([0x80, 0x3F, 0x00, 0xC0, 0x00, 0x3F])),
                                         ("h", "F16", [4], bytes([0x00, 0x3C, 0x00, 0x38, 0x00, 0xC0, 0, 0]))]))
    assert kernrt_b200.safetensors_tensor(p, "b")["dtype"] == "BF16"
    assert kernrt_b200.safetensors_tensor(p, "h")["dtype"] == "F16"


def test_oracle_widening_matches_the_reference_known_answers(oracle):
    # safetensors.rs:471-485 decodes_bfloat16_weights / decodes_float16_weights
    b = np.frombuffer(bytes([0x80, 0x3F, 0x00, 0xC0, 0x00, 0x3F]), np.uint16)
    h = np.frombuffer(bytes([0x00, 0x3C, 0x00, 0x38, 0x00, 0xC0, 0x00, 0x00]), np.uint16)
    assert oracle.st_widen("BF16", b).tolist() == [1.0, -2.0, 0.5]
    assert oracle.st_widen("F16", h).tolist() == [1.0, 0.5, -2.0, 0.0]
    # every non-NaN half: the restated loop equals the exact conversion
    v = np.arange(65536, dtype=np.uint16)
    want = v.view(np.float16).astype(np.float32)
    got = oracle.st_f16_to_f32(v)
    m = ~np.isnan(want)
    assert np.array_equal(got[m].view(np.uint32), want[m].view(np.uint32))
    # NaN keeps its sign and mantissa bits shifted into place
    nan = np.array([0x7C01, 0xFE00], np.uint16)
    assert oracle.st_f16_to_f32(nan).view(np.uint32).tolist() == [0x7F802000, 0xFFC00000]


def test_rejects_header_longer_than_file(st_file):
    # safetensors.rs:487-495
    p = st_file((999).to_bytes(8, "little") + b"{}")
    assert err(p) == "file of 10 bytes is too short for a 1007-byte header"
    p = st_file(b"\x01\x02")
    assert err(p) == "file of 2 bytes is too short for a 8-byte header"


def test_rejects_offsets_that_do_not_match_shape(st_file):
    # safetensors.rs:497-511: two elements of shape, one of payload
    p = st_file(_data.safetensors_raw(b'{"w": {"dtype": "F32", "shape": [2], "data_offsets": [0, 4]}}', f32b(1.0)))
    assert err(p) == 'tensor "w" has byte range 0..4 that does not match its shape'


def test_rejects_offsets_past_end_of_file(st_file):
    # safetensors.rs:513-526
    p = st_file(_data.safetensors_raw(b'{"w": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}', f32b(1.0)))
    assert "has byte range 0..8" in err(p)


def test_rejects_invalid_json(st_file):
    # safetensors.rs:528-536
    assert err(st_file(_data.safetensors_raw(b"not json"))).startswith("invalid header JSON: ")
    for bad in [b'{"w": 1,}', b'{"w": [1, 2,]}', b"{'w': 1}", b'{"w": 1} x', b'{"w": "\\ud800"}',
                b'{"w": "\\udc00"}', b'{"w": 01}', b'{"w": "a\x01"}', b'{"w": "\xff"}', b"[" * 200 + b"]" * 200]:
        assert err(st_file(_data.safetensors_raw(bad))).startswith("invalid header JSON: "), bad


@pytest.mark.parametrize("header,message", [
    (b'[]', "invalid header: top level is not an object"),
    (b'{"w": 3}', 'invalid header: tensor "w" is not an object'),
    (b'{"w": {"shape": [1], "data_offsets": [0, 4]}}', 'invalid header: tensor "w" has no dtype'),
    (b'{"w": {"dtype": 5, "shape": [1], "data_offsets": [0, 4]}}', 'invalid header: tensor "w" has no dtype'),
    (b'{"w": {"dtype": "F32", "data_offsets": [0, 4]}}', 'invalid header: tensor "w" has no shape array'),
    (b'{"w": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}',
     'invalid header: tensor "w" has a non-integer shape'),
    (b'{"w": {"dtype": "F32", "shape": [1.0], "data_offsets": [0, 4]}}',
     'invalid header: tensor "w" has a non-integer shape'),
    (b'{"w": {"dtype": "F32", "shape": [1]}}', 'invalid header: tensor "w" has no data_offsets'),
    (b'{"w": {"dtype": "F32", "shape": [1], "data_offsets": [0]}}',
     'invalid header: tensor "w" needs two integer data_offsets'),
    (b'{"w": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}}',
     'tensor "w" has byte range 4..0 that does not match its shape'),
    (b'{"w": {"dtype": "F32", "shape": [4294967296, 4294967296], "data_offsets": [0, 4]}}',
     'tensor "w" has byte range 0..4 that does not match its shape'),
])
def test_rejects_malformed_entries(st_file, header, message):
    assert err(st_file(_data.safetensors_raw(header, f32b(1.0)))) == message


def test_entries_are_checked_in_key_order_and_duplicates_keep_the_last(st_file):
    # the reference's JSON map is sorted by key; a later duplicate replaces the earlier
    h = b'{"b": 3, "a": {"dtype": "X"}}'
    assert err(st_file(_data.safetensors_raw(h)), "b") == 'unsupported dtype "X" (F32, BF16 and F16 are read)'
    h = b'{"w": {"dtype": "F32", "shape": [9], "data_offsets": [0, 36]}, ' \
        b'"w": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}}'
    assert kernrt_b200.safetensors_tensor(st_file(_data.safetensors_raw(h, f32b(1.0))), "w")["shape"] == (1,)


def test_names_with_escapes(st_file):
    h = '{"emb\\u00e9\\ud83d\\ude00\\"x": {"dtype": "BF16", "shape": [2, 2], "data_offsets": [0, 8]}}'.encode()
    p = st_file(_data.safetensors_raw(h, bytes(8)))
    assert kernrt_b200.safetensors_tensor(p, "embé\U0001F600\"x")["shape"] == (2, 2)
