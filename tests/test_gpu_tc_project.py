"""Tolerance-mode projections on the tensor cores (kernrt_cuda_set_exact(0)).

The reference's dot (reference.rs:73-79) is one f32 accumulator left to right;
the tensor-core path reorders that sum, so it is held to a tolerance instead of
bit parity:

* per output, |g - r| <= 1e-5 * sum_k |W[o,k] x[r,k]| against the oracle's
  exact projection (the split x = hi + lo keeps ~16 bits of each activation,
  each product is exact in f32, the accumulation is f32);
* on a small two-layer model prefilled through the trait ops, the logits of
  the last row within 1e-3 of the exact path's and the same argmax: the bar the
  reference sets for a non-oracle backend (tests/backends.rs:129-148).

Matrices that are not bf16, and calls of fewer than 16 rows, stay exact.
"""
import numpy as np
import pytest

import kernrt_b200
from tests import _data
from tests._parity import assert_bits_equal

pytestmark = pytest.mark.gpu


def check_close(got, want, w, x, what):
    bound = 1e-5 * (np.abs(x.astype(np.float64)) @ np.abs(w.astype(np.float64)).T) + 1e-30
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    worst = float((err / bound).max())
    assert worst <= 1.0, f"{what}: error {worst:.3g}x the bound (max abs error {err.max():.3g})"


# tile edges in every direction: outputs not a multiple of 128, inputs not a
# multiple of 64, rows not a multiple of 64; K from 64 to 8192
SHAPES = [(2048, 2048, 512), (256, 512, 100), (130, 72, 64), (64, 96, 16), (300, 1032, 17), (8192, 2048, 64),
          (2048, 8192, 128), (1000, 576, 33)]


@pytest.mark.parametrize("out_dim,in_dim,rows", SHAPES)
def test_tc_project_within_tolerance(gpu, oracle, out_dim, in_dim, rows):
    w = _data.bf16_table(out_dim, in_dim, 700 + in_dim, 0.05)
    x = _data.lcg_normal(rows * in_dim, 701 + rows).reshape(rows, in_dim)
    m = gpu.prepare_matrix(kernrt_b200.BF16, w, None, out_dim, in_dim)
    hx, hy = gpu.upload(x), gpu.alloc(rows * out_dim)
    gpu.set_exact(False)
    try:
        gpu.project(m, hx, hy, rows)
        got = gpu.read(hy, rows * out_dim).reshape(rows, out_dim)
    finally:
        gpu.set_exact(True)
    want = oracle.project(oracle.BF16, w, None, out_dim, in_dim, x)
    check_close(got, want, oracle.bf16_to_f32(w), x, f"tc project {out_dim}x{in_dim}, {rows} rows")


def test_tc_project_sets_share_one_split(gpu, oracle):
    """project_qkv / project_gate_up in tolerance mode: x split once, one
    tensor-core launch per matrix."""
    dim, kv, hidden, rows = 512, 256, 1024, 80
    x = _data.lcg_normal(rows * dim, 720).reshape(rows, dim)
    hx = gpu.upload(x)
    ws = {n: _data.bf16_table(o, dim, 721 + i, 0.05) for i, (n, o) in enumerate([("q", dim), ("k", kv), ("v", kv),
                                                                                 ("g", hidden), ("u", hidden)])}
    ms = {n: gpu.prepare_matrix(kernrt_b200.BF16, w, None, w.shape[0], dim) for n, w in ws.items()}
    ys = {n: gpu.alloc(rows * w.shape[0]) for n, w in ws.items()}
    gpu.set_exact(False)
    try:
        gpu.project_qkv(ms["q"], ms["k"], ms["v"], hx, ys["q"], ys["k"], ys["v"], rows)
        gpu.project_gate_up(ms["g"], ms["u"], hx, ys["g"], ys["u"], rows)
        got = {n: gpu.read(ys[n], rows * w.shape[0]).reshape(rows, w.shape[0]) for n, w in ws.items()}
    finally:
        gpu.set_exact(True)
    for n, w in ws.items():
        want = oracle.project(oracle.BF16, w, None, w.shape[0], dim, x)
        check_close(got[n], want, oracle.bf16_to_f32(w), x, f"tc project set ({n})")


def test_tolerance_mode_small_calls_and_other_storages(gpu, oracle):
    """Decode-sized bf16 calls (1-4 rows) sum each output across a warp (within
    the bound); 5-15 rows and Q8_0 matrices stay bit-exact."""
    out_dim, in_dim = 256, 512
    w = _data.bf16_table(out_dim, in_dim, 730, 0.05)
    m = gpu.prepare_matrix(kernrt_b200.BF16, w, None, out_dim, in_dim)
    codes, scales = _data.q8_table(out_dim, in_dim, 731)
    mq = gpu.prepare_matrix(kernrt_b200.Q8_0, codes, scales, out_dim, in_dim)
    gpu.set_exact(False)
    try:
        for rows in (1, 4, 5, 15):
            x = _data.lcg_normal(rows * in_dim, 732 + rows).reshape(rows, in_dim)
            hx, hy = gpu.upload(x), gpu.alloc(rows * out_dim)
            gpu.project(m, hx, hy, rows)
            got = gpu.read(hy, rows * out_dim).reshape(rows, out_dim)
            want = oracle.project(oracle.BF16, w, None, out_dim, in_dim, x)
            if rows <= 4:
                check_close(got, want, oracle.bf16_to_f32(w), x, f"bf16, {rows} rows (warp sums)")
            else:
                assert_bits_equal(got, want, f"bf16, {rows} rows")
        rows = 64
        x = _data.lcg_normal(rows * in_dim, 740).reshape(rows, in_dim)
        hx, hy = gpu.upload(x), gpu.alloc(rows * out_dim)
        gpu.project(mq, hx, hy, rows)
        assert_bits_equal(gpu.read(hy, rows * out_dim).reshape(rows, out_dim),
                          oracle.project(oracle.Q8_0, codes, scales, out_dim, in_dim, x), "q8_0, 64 rows")
    finally:
        gpu.set_exact(True)


@pytest.mark.parametrize("out_dim,in_dim,rows", [(2048, 2048, 1), (8192, 2048, 2), (2048, 8192, 1), (130, 72, 4),
                                                 (300, 1032, 3), (49152, 576, 1)])
def test_tolerance_decode_projection_within_bound(gpu, oracle, out_dim, in_dim, rows):
    w = _data.bf16_table(out_dim, in_dim, 760 + in_dim, 0.05)
    x = _data.lcg_normal(rows * in_dim, 761 + rows).reshape(rows, in_dim)
    m = gpu.prepare_matrix(kernrt_b200.BF16, w, None, out_dim, in_dim)
    hx, hy = gpu.upload(x), gpu.alloc(rows * out_dim)
    gpu.set_exact(False)
    try:
        gpu.project(m, hx, hy, rows)
        got = gpu.read(hy, rows * out_dim).reshape(rows, out_dim)
    finally:
        gpu.set_exact(True)
    want = oracle.project(oracle.BF16, w, None, out_dim, in_dim, x)
    check_close(got, want, oracle.bf16_to_f32(w), x, f"decode project {out_dim}x{in_dim}, {rows} rows")


def test_tolerance_decode_sets_are_one_launch(gpu, oracle):
    dim, kv, hidden, rows = 512, 256, 1024, 1
    x = _data.lcg_normal(rows * dim, 770).reshape(rows, dim)
    hx = gpu.upload(x)
    ws = {n: _data.bf16_table(o, dim, 771 + i, 0.05) for i, (n, o) in enumerate([("q", dim), ("k", kv), ("v", kv),
                                                                                 ("g", hidden), ("u", hidden)])}
    ms = {n: gpu.prepare_matrix(kernrt_b200.BF16, w, None, w.shape[0], dim) for n, w in ws.items()}
    ys = {n: gpu.alloc(rows * w.shape[0]) for n, w in ws.items()}
    gpu.set_exact(False)
    try:
        gpu.synchronize()
        n0 = kernrt_b200.kernel_launches()
        gpu.project_qkv(ms["q"], ms["k"], ms["v"], hx, ys["q"], ys["k"], ys["v"], rows)
        gpu.project_gate_up(ms["g"], ms["u"], hx, ys["g"], ys["u"], rows)
        gpu.synchronize()
        assert kernrt_b200.kernel_launches() - n0 == 2
        got = {n: gpu.read(ys[n], rows * w.shape[0]).reshape(rows, w.shape[0]) for n, w in ws.items()}
    finally:
        gpu.set_exact(True)
    for n, w in ws.items():
        want = oracle.project(oracle.BF16, w, None, w.shape[0], dim, x)
        check_close(got[n], want, oracle.bf16_to_f32(w), x, f"decode set ({n})")


def _prefill_logits(b, exact, rows=64, dim=256, n_heads=4, n_kv=2, hidden=512, vocab=1000, n_layers=2, seed=750):
    """A two-layer Llama-style prefill through the trait ops in the driver's
    order (llama.rs prefill), bf16 weights; the logits of the last row."""
    head = dim // n_heads
    kv_dim = n_kv * head
    rng = np.random.default_rng(seed)

    def mat(o, i):
        w = _data.bf16_table(o, i, int(rng.integers(1 << 30)), 1.0 / np.sqrt(i))
        return b.prepare_matrix(kernrt_b200.BF16, w, None, o, i)

    emb = _data.bf16_table(vocab, dim, int(rng.integers(1 << 30)), 0.5)
    b.prepare_embedding(kernrt_b200.BF16, emb, None, vocab, dim)
    cls = b.prepare_matrix(kernrt_b200.BF16, emb, None, vocab, dim)
    layers = [dict(q=mat(dim, dim), k=mat(kv_dim, dim), v=mat(kv_dim, dim), o=mat(dim, dim), g=mat(hidden, dim),
                   u=mat(hidden, dim), d=mat(dim, hidden)) for _ in range(n_layers)]
    b.kv_prepare(n_layers, kv_dim, rows)
    norm_w = b.upload((1 + 0.1 * rng.standard_normal(dim)).astype(np.float32))
    x, xb, o = (b.alloc(rows * dim) for _ in range(3))
    q, att_o = b.alloc(rows * dim), b.alloc(rows * dim)
    k, v = b.alloc(rows * kv_dim), b.alloc(rows * kv_dim)
    g, u = b.alloc(rows * hidden), b.alloc(rows * hidden)
    att = b.alloc(rows * n_heads * rows)
    last, logits = b.alloc(dim), b.alloc(vocab)
    tokens = rng.integers(0, vocab, rows)
    pos = list(range(rows))
    b.set_exact(exact)
    for r, t in enumerate(tokens):
        b.embed(int(t), x, r * dim)
    for li, L in enumerate(layers):
        b.rms_norm(xb, x, norm_w, rows, dim, 1e-5)
        b.project_qkv(L["q"], L["k"], L["v"], xb, q, k, v, rows)
        b.rope(q, k, dim, kv_dim, rows, pos, head, 1e4, False)
        b.kv_write(li, pos, k, v, rows)
        b.attention(q, att_o, att, li, [(0, r, 0, 0) for r in pos], n_heads, n_heads // n_kv, head, kv_dim, rows)
        b.project(L["o"], att_o, o, rows)
        b.add_in_place(x, o, rows * dim)
        b.rms_norm(xb, x, norm_w, rows, dim, 1e-5)
        b.project_gate_up(L["g"], L["u"], xb, g, u, rows)
        b.silu_mul(g, u, rows * hidden)
        b.project(L["d"], g, o, rows)
        b.add_in_place(x, o, rows * dim)
    b.copy(x, (rows - 1) * dim, last, 0, dim)
    b.rms_norm(xb, last, norm_w, 1, dim, 1e-5)
    b.logits(cls, xb, logits)
    out = b.read(logits, vocab)
    b.set_exact(True)
    return out


def test_tc_prefill_logits_meet_the_reference_bar():
    """tests/backends.rs:129-148's bar for a non-oracle backend: logits within
    1e-3 of the exact path (bit-identical to the reference backend's
    projections) and the same argmax."""
    with kernrt_b200.CudaBackend(0) as b:
        want = _prefill_logits(b, exact=True)
    with kernrt_b200.CudaBackend(0) as b:
        got = _prefill_logits(b, exact=False)
    diff = float(np.abs(got.astype(np.float64) - want).max())
    assert diff <= 1e-3, f"tolerance-mode logits differ by {diff}"
    assert int(np.argmax(got)) == int(np.argmax(want))


def test_tolerance_decode_logits_meet_the_reference_bar():
    """The same bar for a decode-sized pass (4 rows: every projection and the
    classifier on the warp-sum kernel)."""
    with kernrt_b200.CudaBackend(0) as b:
        want = _prefill_logits(b, exact=True, rows=4)
    with kernrt_b200.CudaBackend(0) as b:
        got = _prefill_logits(b, exact=False, rows=4)
    diff = float(np.abs(got.astype(np.float64) - want).max())
    assert diff <= 1e-3, f"tolerance-mode logits differ by {diff}"
    assert int(np.argmax(got)) == int(np.argmax(want))
