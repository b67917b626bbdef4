"""Pin the CPU oracle against KernRT's own known-answer tests (no GPU).

KernRT is Rust and cannot be built here, so the oracle (oracle/kernrt_oracle.c)
is pinned by restating every known-answer test the reference holds for the
row-op path, each citing its source, plus the committed golden fixtures.
"""
import json
import math
import os

import numpy as np
import pytest

from tests import _data

HERE = os.path.dirname(os.path.abspath(__file__))
f32 = np.float32


def test_lcg_matches_sequential_definition():
    # tests/backends.rs:41-51: the sequential LCG, restated naively.
    state = 12345
    want = []
    for _ in range(1000):
        state = (state * 6364136223846793005 + 1442695040888963407) % (1 << 64)
        want.append(f32(state >> 40) / f32(1 << 24) - f32(0.5))
    got = _data.lcg_uniform(1000, 12345)
    assert np.array_equal(got, np.array(want, np.float32))


# --- src/backends/metal.rs:1926-2280 kernels_match_their_reference --------------

def test_metal_kat_rms_norm(oracle):
    x = np.array([1, 2, 3, 4], f32)
    got = oracle.rms_norm(x[None], np.ones(4, f32), 0.0)[0]
    scale = f32(1.0) / np.sqrt(f32((x * x).sum() / 4))
    assert np.all(np.abs(got - x * scale) < 1e-5)


def test_metal_kat_qk_norm(oracle):
    got = oracle.qk_norm(np.array([[3, 4, 0, 2]], f32), 2, np.ones(2, f32), 0.0)[0]
    assert abs(got[0] - 3 / math.sqrt(12.5)) < 1e-5
    assert abs(got[3] - 2 / math.sqrt(2.0)) < 1e-5


def test_metal_kat_silu_mul(oracle):
    got = oracle.silu_mul(np.array([1, -1], f32), np.array([2, 2], f32))
    silu = lambda v: v / (1 + math.exp(-v))  # noqa: E731
    assert abs(got[0] - silu(1.0) * 2) < 1e-5


def test_metal_kat_copy(oracle):
    a = np.array([7, 8, 9], f32)
    b = np.zeros(3, f32)
    oracle.copy_into(a, 1, b, 0, 2)
    assert list(b[:2]) == [8.0, 9.0]


def test_metal_kat_rope_half(oracle):
    q = np.array([[0.3, -0.7, 1.1, 0.2]], f32)
    got, _ = oracle.rope(q, np.zeros((1, 4), f32), [3], 4, 10000.0, interleaved=False)
    for i in range(2):
        freq = f32(1.0) / np.power(f32(10000.0), f32(2 * i) / f32(4.0))
        s, c = math.sin(3.0 * freq), math.cos(3.0 * freq)
        lo, hi = q[0, i], q[0, i + 2]
        assert abs(got[0, i] - (lo * c - hi * s)) < 1e-5
        assert abs(got[0, i + 2] - (lo * s + hi * c)) < 1e-5


def test_metal_kat_add(oracle):
    got = oracle.add_in_place(np.array([1, 2], f32), np.array([10, 20], f32))
    assert list(got) == [11.0, 22.0]


def test_metal_kat_mul_offsets_same_buffer(oracle):
    ab = np.array([1, 2, 3, 4, 5, 6], f32)
    o = np.zeros(2, f32)
    oracle.mul_into(o, 0, ab, 1, ab, 3, 2)
    assert list(o) == [2 * 4, 3 * 5]


def _conv_kat_inputs():
    x = np.arange(16, dtype=f32) + 1
    kw = np.array([1, 0, 0, 0, 1, 0, 0, 0, 1, 1, 1, 1], f32)
    return x, kw


def test_metal_kat_conv_prefill(oracle):
    x, kw = _conv_kat_inputs()
    got = oracle.conv_prefill(x.reshape(4, 4), kw, 3).ravel()
    assert got[0] == 0.0 and got[4] == 0.0
    assert got[8] == x[0] and got[12] == x[4]
    assert got[3] == x[3]
    assert got[15] == x[7] + x[11] + x[15]


def test_metal_kat_conv_decode_ring(oracle):
    _, kw = _conv_kat_inputs()
    st = np.array([10, 20, 30, 40, 50, 60, 70, 80], f32)
    out, ring = oracle.conv_decode(np.ones(4, f32), kw, st, 3)
    assert out[0] == 10.0
    assert out[3] == 40.0 + 80.0 + 1.0
    assert list(ring) == [50, 60, 70, 80, 1, 1, 1, 1]


# --- src/arch/llm/llama.rs:954-1015 ----------------------------------------------

def test_llama_qk_norm_normalizes_each_head_separately(oracle):
    data = np.array([[3, 0, 0, 0, 0.1, 0.1, 0.1, 0.1]], f32)
    out = oracle.qk_norm(data, 4, np.ones(4, f32), 0.0)[0]
    rms = lambda h: math.sqrt(float((h * h).sum()) / len(h))  # noqa: E731
    assert abs(rms(out[:4]) - 1) < 1e-5 and abs(rms(out[4:]) - 1) < 1e-5
    assert abs(out[0] - 2.0) < 1e-5
    assert np.all(out[1:4] == 0.0)


@pytest.mark.parametrize("interleaved", [True, False])
def test_llama_rope_styles_preserve_norms(oracle, interleaved):
    q = np.array([[0.3, -0.7, 1.1, 0.2, -0.4, 0.9, 0.5, -0.1]], f32)
    out, _ = oracle.rope(q, np.zeros_like(q), [3], 4, 10000.0, interleaved=interleaved)
    ssum = lambda v: float((v.astype(f32) * v.astype(f32)).sum(dtype=f32))  # noqa: E731
    assert abs(ssum(out) - ssum(q)) < 1e-5


# --- src/arch/llm/lfm2.rs:829-866 --------------------------------------------------

def test_lfm2_conv_prefill_matches_stepped_decode(oracle):
    dim, k, rows = 8, 3, 5
    h = np.sin(np.arange(rows * dim, dtype=f32) * f32(0.37)).astype(f32).reshape(rows, dim)
    kw = np.cos(np.arange(dim * k, dtype=f32) * f32(0.11)).astype(f32)
    got = oracle.conv_prefill(h, kw, k)
    state = np.zeros(dim * (k - 1), f32)
    want = np.zeros_like(got)
    for r in range(rows):
        want[r], state = oracle.conv_decode(h[r], kw, state, k)
    assert float(np.abs(got - want).max()) <= 1e-5


# --- src/ops/mod.rs Q8 and bf16 known answers ----------------------------------------

def test_q8_quantization_error_is_half_a_step(oracle):
    # src/ops/mod.rs:557-572
    for seed in range(8):
        x = _data.lcg_uniform(96, 100 + seed)
        q, s, _ = oracle.q8_quantize(x)
        for b, scale in enumerate(s):
            restored = q[b * 32:(b + 1) * 32].astype(f32) * scale
            assert np.all(np.abs(restored - x[b * 32:(b + 1) * 32]) <= scale / 2 + 1e-6)


def test_q8_is_exact_on_step_multiples(oracle):
    # src/ops/mod.rs:577-597
    step = f32(1.0 / 128.0)
    vals = []
    for _ in range(2):
        for lane in range(32):
            kk = 127.0 if lane == 0 else lane - 16.0
            vals.append(f32(kk) * step)
    vals = np.array(vals, f32)
    q, s, _ = oracle.q8_quantize(vals)
    for b, scale in enumerate(s):
        assert scale == step
        assert np.array_equal(q[b * 32:(b + 1) * 32].astype(f32) * scale, vals[b * 32:(b + 1) * 32])


def test_bf16_matrix_reads_rows(oracle):
    # src/ops/mod.rs:545-554
    bits = (np.array([1.0, -2.0, 0.5, 4.0], f32).view(np.uint32) >> 16).astype(np.uint16)
    row = oracle.embed_rows(oracle.BF16, bits, None, 2, 2, [1])[0]
    assert list(row) == [0.5, 4.0]


def test_bf16_bits_round_to_the_stored_width(oracle):
    # src/ops/mod.rs:753-763
    vals = np.array([0.0, 1.0, -1.0, 0.1, 0.123456, 1e-3, -1234.5, 1e20], f32)
    back = oracle.bf16_to_f32(oracle.f32_to_bf16_bits(vals))
    tol = np.abs(vals) * f32(0.0039) + np.finfo(np.float32).tiny
    assert np.all(np.abs(back - vals) <= tol)
    for b in (0x3F80, 0xBF80, 0x0000):
        v = oracle.bf16_to_f32(np.array([b], np.uint16))
        assert oracle.f32_to_bf16_bits(v)[0] == b


def test_f16_conversion_matches_ieee(oracle):
    # src/ops/quant.rs:722-758 is IEEE binary16 RNE for every finite input:
    # check it against numpy's converter over normals, subnormals and overflow.
    vals = np.concatenate([
        _data.lcg_uniform(4000, 3) * f32(1e-2),
        _data.lcg_uniform(1000, 4) * f32(1e-6),
        _data.lcg_uniform(1000, 5) * f32(1e5),
        np.array([0.0, -0.0, 65504.0, 65520.0, 7e4, 5.96e-8, 2.98e-8], f32),
    ]).astype(f32)
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    got = np.array([oracle.f32_to_f16_bits(v) for v in vals], np.uint16)
    assert np.array_equal(got, want)


def test_q8_0x4_round_trip(oracle):
    # quant.rs:124-165 packs, :198-220 de-interleaves; rows decode identically
    # through Q8_0x4::row (:174-190) and the row-major form.
    w = _data.lcg_normal(8 * 64, 11).reshape(8, 64)
    blocks = oracle.q8_0x4_pack(w)
    q, s = oracle.q8_0x4_to_row_major(blocks, 8, 64)
    rows_packed = oracle.embed_rows(oracle.Q8_0X4, blocks, None, 8, 64, np.arange(8))
    rows_major = oracle.embed_rows(oracle.Q8_0, q, s, 8, 64, np.arange(8))
    assert np.array_equal(rows_packed.view(np.uint32), rows_major.view(np.uint32))


# --- committed golden fixtures --------------------------------------------------------

def test_golden_fixtures(oracle):
    """tests/golden/*.json were generated by tests/golden/make_golden.py; the
    oracle must reproduce their bits (guards against libm/compiler drift)."""
    path = os.path.join(HERE, "golden", "golden.json")
    with open(path) as fh:
        g = json.load(fh)
    from tests.golden import make_golden

    fresh = make_golden.compute(oracle)
    for name, want in g["cases"].items():
        got = fresh[name]
        assert got == want, f"golden case {name} drifted"
