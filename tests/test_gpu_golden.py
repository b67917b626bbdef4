"""CUDA outputs against the committed golden digests and KernRT's own GPU
known-answer test (src/backends/metal.rs:1926-2280), through the C ABI."""
import hashlib
import json
import math
import os

import numpy as np
import pytest

import kernrt_b200
from tests.golden import make_golden
from tests._parity import assert_close_rel

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
f32 = np.float32


def _h(*arrays):
    m = hashlib.sha256()
    for a in arrays:
        m.update(np.ascontiguousarray(a).tobytes())
    return m.hexdigest()


def test_cuda_matches_golden_digests(gpu, oracle):
    with open(os.path.join(HERE, "golden", "golden.json")) as fh:
        golden = json.load(fh)["cases"]
    d = make_golden.inputs()
    up = lambda a: gpu.upload(np.ascontiguousarray(a, f32))  # noqa: E731
    got = {}

    x = d["rms_x"]
    o = gpu.alloc(x.size)
    gpu.rms_norm(o, up(x), up(d["rms_w"]), 7, 576, 1e-5)
    got["rms_norm_576"] = _h(gpu.read(o, x.size).reshape(x.shape))

    v = up(d["qk_v"])
    gpu.qk_norm(v, 5, 1024, 128, up(d["qk_w"]), 1e-6)
    got["qk_norm_128"] = _h(gpu.read(v, 5 * 1024).reshape(5, 1024))

    for name, inter in [("rope_half_64", False), ("rope_pair_64", True)]:
        q, k = up(d["rope_q"]), up(d["rope_k"])
        gpu.rope(q, k, 576, 192, 6, d["rope_pos"], 64, 1e5, inter)
        got[name] = _h(gpu.read(q, 6 * 576).reshape(6, 576), gpu.read(k, 6 * 192).reshape(6, 192))

    xc = d["conv_x"]
    o = gpu.alloc(xc.size)
    gpu.conv_prefill(o, up(xc), up(d["conv_w"]), 9, 40, 3)
    got["conv_prefill_k3"] = _h(gpu.read(o, xc.size).reshape(xc.shape))

    xq = d["q8_x"]
    nb = (1000 + 31) // 32
    c, s, h16 = gpu.alloc_bytes(3 * nb * 32), gpu.alloc_bytes(3 * nb * 4), gpu.alloc_bytes(3 * nb * 2)
    gpu.quantize_q8_0(up(xq), 3, 1000, c, s, h16)
    got["q8_quantize"] = _h(gpu.read_bytes(c, 3 * nb * 32, np.int8).reshape(3, -1),
                            gpu.read_bytes(s, 3 * nb * 4, np.float32).reshape(3, -1),
                            gpu.read_bytes(h16, 3 * nb * 2, np.uint16).reshape(3, -1))

    toks = d["emb_tok"]
    for name, kind, data, sc in [("embed_bf16", kernrt_b200.BF16, d["emb_bf16"], None),
                                 ("embed_q8_0", kernrt_b200.Q8_0, d["emb_q8"], d["emb_q8_s"])]:
        gpu.prepare_embedding(kind, data, sc, 64, 96)
        o = gpu.alloc(len(toks) * 96)
        for r, t in enumerate(toks):
            gpu.embed(int(t), o, r * 96)
        got[name] = _h(gpu.read(o, len(toks) * 96).reshape(len(toks), 96))

    for name, digest in golden.items():
        if name == "silu_mul":
            continue  # tolerance, not bits: checked below
        assert got[name] == digest, f"{name}: CUDA output differs from the golden digest"

    g = up(d["silu_g"])
    gpu.silu_mul(g, up(d["silu_u"]), 3000)
    assert_close_rel(gpu.read(g, 3000), oracle.silu_mul(d["silu_g"], d["silu_u"]), what="silu")


def test_metal_known_answers_on_cuda(gpu):
    """The reference's GPU kernel KAT, restated for this backend."""
    up = lambda a: gpu.upload(np.array(a, f32))  # noqa: E731
    x = [1.0, 2.0, 3.0, 4.0]
    o = gpu.alloc(4)
    gpu.rms_norm(o, up(x), up([1, 1, 1, 1]), 1, 4, 0.0)
    got = gpu.read(o, 4)
    scale = 1.0 / math.sqrt(sum(v * v for v in x) / 4)
    assert all(abs(got[i] - x[i] * scale) < 1e-5 for i in range(4))

    vb = up([3.0, 4.0, 0.0, 2.0])
    gpu.qk_norm(vb, 1, 4, 2, up([1, 1]), 0.0)
    got = gpu.read(vb, 4)
    assert abs(got[0] - 3 / math.sqrt(12.5)) < 1e-5 and abs(got[3] - 2 / math.sqrt(2)) < 1e-5

    gb = up([1.0, -1.0])
    gpu.silu_mul(gb, up([2.0, 2.0]), 2)
    assert abs(gpu.read(gb, 2)[0] - 2 / (1 + math.exp(-1))) < 1e-5

    a, b = up([7, 8, 9]), gpu.alloc(3)
    gpu.copy(a, 1, b, 0, 2)
    assert list(gpu.read(b, 2)) == [8.0, 9.0]

    q = [0.3, -0.7, 1.1, 0.2]
    qb, kb = up(q), up([0, 0, 0, 0])
    gpu.rope(qb, kb, 4, 4, 1, [3], 4, 10000.0, False)
    got = gpu.read(qb, 4)
    for i in range(2):
        freq = f32(1.0) / np.power(f32(10000.0), f32(2 * i) / f32(4.0))
        s, c = math.sin(3.0 * freq), math.cos(3.0 * freq)
        assert abs(got[i] - (q[i] * c - q[i + 2] * s)) < 1e-5
        assert abs(got[i + 2] - (q[i] * s + q[i + 2] * c)) < 1e-5

    d = up([1, 2])
    gpu.add_in_place(d, up([10, 20]), 2)
    assert list(gpu.read(d, 2)) == [11.0, 22.0]

    ab, o = up([1, 2, 3, 4, 5, 6]), gpu.alloc(2)
    gpu.mul(o, 0, ab, 1, ab, 3, 2)
    assert list(gpu.read(o, 2)) == [8.0, 15.0]

    xs = [float(i + 1) for i in range(16)]
    kw = up([1, 0, 0, 0, 1, 0, 0, 0, 1, 1, 1, 1])
    co = gpu.alloc(16)
    gpu.conv_prefill(co, up(xs), kw, 4, 4, 3)
    got = gpu.read(co, 16)
    assert got[0] == 0 and got[4] == 0 and got[8] == xs[0] and got[12] == xs[4]
    assert got[3] == xs[3] and got[15] == xs[7] + xs[11] + xs[15]

    st = up([10, 20, 30, 40, 50, 60, 70, 80])
    orow = gpu.alloc(4)
    gpu.conv_decode(orow, up([1, 1, 1, 1]), kw, st, 4, 3)
    got = gpu.read(orow, 4)
    assert got[0] == 10.0 and got[3] == 121.0
    assert list(gpu.read(st, 8)) == [50, 60, 70, 80, 1, 1, 1, 1]
