"""The drop-in path on KernRT's real call sequences.

KernRT's drivers call the row ops one trait method at a time, interleaved with
contractions (src/arch/llm/llama.rs:734-770, lfm2.rs:584-624).  The backend
defers one op and fuses it with the next when they form one of the driver's
pairs: embed x R -> rms_norm, add_in_place -> rms_norm, qk_norm(q), qk_norm(k)
-> rope, rope -> kv_write (tests/test_gpu_contract.py), and per-row mul runs.
These tests replay those sequences (with the contractions' outputs uploaded in
their place) and require the oracle's bits and the fused launch counts.
"""
import numpy as np
import pytest

import kernrt_b200
from tests import _data
from tests._parity import assert_bits_equal, assert_close_rel

pytestmark = pytest.mark.gpu
f32 = np.float32


def test_llama_layer_sequence_fuses_and_matches_oracle(gpu, oracle):
    R, dim, q_dim, kv_dim, head, hidden, vocab = 48, 256, 256, 128, 64, 512, 100
    eps, theta = 1e-6, 1e6
    rng = np.random.default_rng(21)
    table = _data.bf16_table_fast(vocab, dim, 22)
    tokens = rng.integers(0, vocab, R).astype(np.int32)
    pos = np.arange(R, dtype=np.uint64) + 7
    w = {n: (1 + 0.1 * rng.standard_normal(n_)).astype(f32)
         for n, n_ in [("att", dim), ("ffn", dim), ("next", dim), ("q", head), ("k", head)]}
    q0 = rng.standard_normal((R, q_dim), dtype=f32)
    k0 = rng.standard_normal((R, kv_dim), dtype=f32)
    o1 = rng.standard_normal((R, dim), dtype=f32)
    o2 = rng.standard_normal((R, dim), dtype=f32)
    g0 = rng.standard_normal((R, hidden), dtype=f32)
    u0 = rng.standard_normal((R, hidden), dtype=f32)

    gpu.prepare_embedding(kernrt_b200.BF16, table, None, vocab, dim)
    hw = {n: gpu.upload(v) for n, v in w.items()}
    x, xb1, xb2, xb3 = (gpu.alloc(R * dim) for _ in range(4))
    q, k, o, oo, g, u = (gpu.upload(a) for a in (q0, k0, o1, o2, g0, u0))
    gpu.synchronize()
    n0 = kernrt_b200.kernel_launches()
    for r, t in enumerate(tokens):                       # llama.rs:734-736
        gpu.embed(int(t), x, r * dim)
    gpu.rms_norm(xb1, x, hw["att"], R, dim, eps)         # :740, fuses with the embeds
    gpu.qk_norm(q, R, q_dim, head, hw["q"], eps)         # :744-749
    gpu.qk_norm(k, R, kv_dim, head, hw["k"], eps)
    gpu.rope(q, k, q_dim, kv_dim, R, pos, head, theta, False)  # :754, fuses with both norms
    gpu.add_in_place(x, o, R * dim)                      # :762
    gpu.rms_norm(xb2, x, hw["ffn"], R, dim, eps)         # :765, fuses with the add
    gpu.silu_mul(g, u, R * hidden)                       # :767
    gpu.add_in_place(x, oo, R * dim)                     # :769
    gpu.rms_norm(xb3, x, hw["next"], R, dim, eps)        # next layer's :740, fuses
    gpu.synchronize()
    launches = kernrt_b200.kernel_launches() - n0
    assert launches == 5, f"expected 5 fused launches, saw {launches}"

    # The oracle runs the same ops unfused, in order.
    xo = oracle.embed_rows(oracle.BF16, table, None, vocab, dim, tokens)
    want_xb1 = oracle.rms_norm(xo, w["att"], eps)
    wq = oracle.qk_norm(q0, head, w["q"], eps)
    wk = oracle.qk_norm(k0, head, w["k"], eps)
    wq, wk = oracle.rope(wq, wk, pos, head, theta)
    xo = oracle.add_in_place(xo, o1)
    want_xb2 = oracle.rms_norm(xo, w["ffn"], eps)
    want_g = oracle.silu_mul(g0, u0)
    xo = oracle.add_in_place(xo, o2)
    want_xb3 = oracle.rms_norm(xo, w["next"], eps)
    got = lambda h, shape: gpu.read(h, int(np.prod(shape))).reshape(shape)  # noqa: E731
    assert_bits_equal(got(xb1, (R, dim)), want_xb1, "xb (attention norm)")
    assert_bits_equal(got(q, (R, q_dim)), wq, "q")
    assert_bits_equal(got(k, (R, kv_dim)), wk, "k")
    assert_bits_equal(got(xb2, (R, dim)), want_xb2, "xb (ffn norm)")
    assert_bits_equal(got(xb3, (R, dim)), want_xb3, "xb (next layer)")
    assert_bits_equal(got(x, (R, dim)), xo, "x (residual stream)")
    assert_close_rel(got(g, (R, hidden)), want_g, what="SwiGLU")


def test_lfm2_conv_sequence_batches_per_row_muls(gpu, oracle):
    R, dim, k = 40, 96, 3
    rng = np.random.default_rng(23)
    bcx = rng.standard_normal((R, 3 * dim), dtype=f32)
    kern = (0.3 * rng.standard_normal(dim * k)).astype(f32)
    ring0 = rng.standard_normal((k - 1) * dim, dtype=f32)
    hb, hk, ring = gpu.upload(bcx), gpu.upload(kern), gpu.upload(ring0)
    h, co, cy = gpu.alloc(R * dim), gpu.alloc(R * dim), gpu.alloc(R * dim)
    gpu.synchronize()
    n0 = kernrt_b200.kernel_launches()
    for r in range(R):                                   # lfm2.rs:586-596
        gpu.mul(h, r * dim, hb, r * 3 * dim, hb, r * 3 * dim + 2 * dim, dim)
    gpu.conv_prefill(co, h, hk, R, dim, k)               # :599
    take = min(R, k - 1)
    gpu.copy(h, (R - take) * dim, ring, (k - 1 - take) * dim, take * dim)  # :601-610
    for r in range(R):                                   # :612-622
        gpu.mul(cy, r * dim, hb, r * 3 * dim + dim, co, r * dim, dim)
    gpu.synchronize()
    assert kernrt_b200.kernel_launches() - n0 == 3  # mul run, conv, mul run (the copy is a memcpy)
    want_cy, want_ring = oracle.lfm2_conv_block(bcx, kern, ring0, k)
    assert_bits_equal(gpu.read(cy, R * dim).reshape(R, dim), want_cy, "cy")
    assert_bits_equal(gpu.read(ring, (k - 1) * dim), want_ring, "ring")


def test_patterns_that_do_not_match_still_run_in_order(gpu, oracle):
    """Near misses of every pattern fall back to the unfused ops, in order."""
    R, dim, head = 6, 64, 16
    rng = np.random.default_rng(24)
    table = _data.bf16_table_fast(20, dim, 25)
    gpu.prepare_embedding(kernrt_b200.BF16, table, None, 20, dim)
    w = gpu.upload(np.ones(dim, f32))
    x, xb = gpu.alloc(R * dim + dim), gpu.alloc(R * dim)
    # embeds with a gap (row 0 at offset dim): no fusion, same result
    toks = [3, 1, 4, 1, 5, 9]
    for r, t in enumerate(toks):
        gpu.embed(t, x, (r + 1) * dim)
    gpu.rms_norm(xb, x, w, R, dim, 1e-5)
    xs = np.zeros((R + 1, dim), f32)
    xs[1:] = oracle.embed_rows(oracle.BF16, table, None, 20, dim, toks)
    assert_bits_equal(gpu.read(xb, R * dim).reshape(R, dim), oracle.rms_norm(xs[:R], np.ones(dim, f32), 1e-5), "gap")
    # add into a different buffer than the one normalised
    a0 = rng.standard_normal((R, dim), dtype=f32)
    b0 = rng.standard_normal((R, dim), dtype=f32)
    ha, hb2, out = gpu.upload(a0), gpu.upload(b0), gpu.alloc(R * dim)
    gpu.add_in_place(ha, hb2, R * dim)
    gpu.rms_norm(out, hb2, w, R, dim, 1e-5)
    assert_bits_equal(gpu.read(out, R * dim).reshape(R, dim), oracle.rms_norm(b0, np.ones(dim, f32), 1e-5), "norm")
    assert_bits_equal(gpu.read(ha, R * dim).reshape(R, dim), a0 + b0, "add")
    # qk_norm over more rows than rope rotates
    q0 = rng.standard_normal((R, dim), dtype=f32)
    k0 = rng.standard_normal((R, dim), dtype=f32)
    hq, hk = gpu.upload(q0), gpu.upload(k0)
    wq = rng.standard_normal(head).astype(f32)
    gpu.qk_norm(hq, R, dim, head, gpu.upload(wq), 1e-6)
    gpu.rope(hq, hk, dim, dim, R, [0, 1, 2], head, 1e4, False)
    wantq = oracle.qk_norm(q0, head, wq, 1e-6)
    rq, rk = oracle.rope(wantq[:3], k0[:3], [0, 1, 2], head, 1e4)
    gotq = gpu.read(hq, R * dim).reshape(R, dim)
    assert_bits_equal(gotq[:3], rq, "rotated rows")
    assert_bits_equal(gotq[3:], wantq[3:], "normalised only")
