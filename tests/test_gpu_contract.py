"""Device contractions against the oracle (reference.rs:73-79, 151-159,
259-306, 402-482): projections, logits and the key/value cache write are
bit-identical to the reference backend's sequential dot; attention differs only
through CUDA's expf, held to |g - r| <= 1e-5 * max|V| for the outputs and the
SwiGLU tolerance (1e-5 relative) for the softmax weights."""
import numpy as np
import pytest

import kernrt_b200
from tests import _data
from tests._parity import assert_bits_equal, assert_close_rel

pytestmark = pytest.mark.gpu
f32 = np.float32


def weights(kind, out_dim, in_dim, seed, oracle):
    """(device kind, host data, scales, oracle kind) for W [out_dim, in_dim]."""
    if kind == "f32":
        return kernrt_b200.F32, _data.lcg_normal(out_dim * in_dim, seed, 0.0, 0.05).reshape(out_dim, in_dim), None, \
            oracle.F32
    if kind == "bf16":
        return kernrt_b200.BF16, _data.bf16_table(out_dim, in_dim, seed, 0.05), None, oracle.BF16
    codes, scales = _data.q8_table(out_dim, in_dim, seed)
    if kind == "q8_0":
        return kernrt_b200.Q8_0, codes, scales, oracle.Q8_0
    w = oracle.embed_rows(oracle.Q8_0, codes, scales, out_dim, in_dim, np.arange(out_dim, dtype=np.int32))
    blocks = oracle.q8_0x4_pack(w)
    return kernrt_b200.Q8_0X4, blocks, None, oracle.Q8_0X4


# tiled kernel for in_dim % 8 == 0 (% 32 for Q8_0), edges in every direction,
# decode (1 row) and prefill (>= 64 rows) tiles, the scalar kernel otherwise
SHAPES = [(96, 64, 1), (2048, 2048, 1), (256, 512, 100), (130, 72, 5), (64, 32, 64), (33, 36, 3), (7, 8, 70),
          (100, 1152, 2), (40, 640, 3), (3000, 1024, 4), (77, 8, 1), (64, 96, 2),
          (5000, 1280, 1), (64, 2560, 2),  # 512- and 1024-column GEMV chunks, partial last chunks
          (64, 1032, 1), (40, 2056, 1)]  # single rows: 16-column steps, then a last chunk of 8 columns


@pytest.mark.parametrize("kind", ["f32", "bf16", "q8_0", "q8_0x4"])
@pytest.mark.parametrize("out_dim,in_dim,rows", SHAPES)
def test_project_matches_reference_dot(gpu, oracle, kind, out_dim, in_dim, rows):
    if kind.startswith("q8") and in_dim % 32:
        pytest.skip("Q8_0 rows are whole 32-element blocks")
    if kind == "q8_0x4" and out_dim % 4:
        pytest.skip("Q8_0x4 holds a multiple of four rows")
    dk, data, scales, ok = weights(kind, out_dim, in_dim, 90 + in_dim, oracle)
    x = _data.lcg_normal(rows * in_dim, 91 + rows).reshape(rows, in_dim)
    m = gpu.prepare_matrix(dk, data, scales, out_dim, in_dim)
    hx, hy = gpu.upload(x), gpu.alloc(rows * out_dim)
    gpu.project(m, hx, hy, rows)
    want = oracle.project(ok, data, scales, out_dim, in_dim, x)
    assert_bits_equal(gpu.read(hy, rows * out_dim).reshape(rows, out_dim), want, f"project {kind}")


def test_logits_is_the_classifier_over_row_zero(gpu, oracle):
    vocab, dim = 3000, 256
    table = _data.bf16_table(vocab, dim, 95)
    x = _data.lcg_normal(3 * dim, 96).reshape(3, dim)
    m = gpu.prepare_matrix(kernrt_b200.BF16, table, None, vocab, dim)
    hx, hy = gpu.upload(x), gpu.alloc(vocab)
    gpu.logits(m, hx, hy)
    want = oracle.project(oracle.BF16, table, None, vocab, dim, x[:1])
    assert_bits_equal(gpu.read(hy, vocab), want[0], "logits")


def attention_case(gpu, oracle, n_layers, n_heads, n_kv, head, seq_len, layer, writes, windows, seed, exact=True):
    kv_dim = n_kv * head
    kv_mul = n_heads // n_kv
    gpu.kv_prepare(n_layers, kv_dim, seq_len)
    kc = np.zeros(n_layers * seq_len * kv_dim, f32)
    vc = np.zeros_like(kc)
    for i, (lay, slots) in enumerate(writes):
        rows = len(slots)
        k = _data.lcg_normal(rows * kv_dim, seed + 2 * i).reshape(rows, kv_dim)
        v = _data.lcg_normal(rows * kv_dim, seed + 2 * i + 1).reshape(rows, kv_dim)
        hk, hv = gpu.upload(k), gpu.upload(v)
        gpu.kv_write(lay, slots, hk, hv, rows)
        oracle.kv_write(kc, vc, kv_dim, seq_len, lay, slots, k, v, rows)
    width = n_heads * head
    q = _data.lcg_normal(len(windows) * width, seed + 50).reshape(len(windows), width)
    hq, ho = gpu.upload(q), gpu.alloc(len(windows) * width)
    ha = gpu.alloc(len(windows) * n_heads * seq_len)
    gpu.set_exact(exact)
    try:
        gpu.attention(hq, ho, ha, layer, windows, n_heads, kv_mul, head, kv_dim, seq_len)
    finally:
        gpu.set_exact(True)
    want_o, want_a = oracle.attention(q, kc, vc, layer, windows, n_heads, kv_mul, head, kv_dim, seq_len)
    got_o = gpu.read(ho, len(windows) * width).reshape(want_o.shape)
    got_a = gpu.read(ha, want_a.size).reshape(want_a.shape)
    bound = 1e-5 * float(np.abs(vc).max())
    err = np.abs(got_o.astype(np.float64) - want_o)
    assert err.max() <= bound, f"attention out: max error {err.max()} above {bound}"
    assert_close_rel(got_a, want_a, what="attention weights")


def test_attention_decode_and_gqa(gpu, oracle):
    # one query at position 40 over slots 0..40, 8 query heads on 2 kv heads
    attention_case(gpu, oracle, 2, 8, 2, 64, 128, 1, [(1, list(range(41))), (0, [3, 4])], [(0, 40, 0, 0)], 300)


def test_attention_prefill_causal_rows(gpu, oracle):
    rows = 37
    wins = [(0, r, 0, 0) for r in range(rows)]
    attention_case(gpu, oracle, 1, 4, 4, 32, 64, 0, [(0, list(range(rows)))], wins, 310)


def test_attention_prefill_row_tiles_with_gqa(gpu, oracle):
    """70 causal rows (row blocks of 16 with a ragged last one), 8 query heads
    on 2 key/value heads: the row-tiled scores share each key tile."""
    rows = 70
    wins = [(0, r, 0, 0) for r in range(rows)]
    attention_case(gpu, oracle, 2, 8, 2, 64, 128, 1, [(1, list(range(rows)))], wins, 315)


def test_attention_prefill_row_tiles_long_windows(gpu, oracle):
    """260 causal rows of head size 64 (value tiles of 64 positions, a 48 KB
    tile set past the default shared-memory limit) and 40 rows of 128."""
    wins = [(0, r, 0, 0) for r in range(260)]
    attention_case(gpu, oracle, 1, 2, 2, 64, 512, 0, [(0, list(range(260)))], wins, 316)
    wins = [(0, 100 + r, 0, 0) for r in range(40)]
    attention_case(gpu, oracle, 1, 2, 1, 128, 256, 0, [(0, list(range(140)))], wins, 317)


def test_attention_rows_sharing_a_prefix_and_start(gpu, oracle):
    """Rows with one shared range and one start, their own last slots: the same
    position map, so the row-tiled scores apply across the shared range."""
    wins = [(40, 40 + r, 0, 24) for r in range(20)]
    attention_case(gpu, oracle, 1, 4, 4, 32, 96, 0, [(0, list(range(96)))], wins, 318)


def test_attention_shared_range_and_window_start(gpu, oracle):
    # rows attending a shared prefix [0, 6) plus their own sliding range
    wins = [(10, 12, 0, 6), (11, 14, 0, 6), (20, 20, 2, 5)]
    attention_case(gpu, oracle, 3, 6, 3, 16, 32, 2, [(2, list(range(32)))], wins, 320)


TOL_CASES = {
    "decode_gqa": (2, 8, 2, 64, 128, 1, [(1, list(range(41))), (0, [3, 4])], [(0, 40, 0, 0)], 340),
    "prefill_causal": (1, 4, 4, 32, 64, 0, [(0, list(range(37)))], [(0, r, 0, 0) for r in range(37)], 341),
    "shared_range": (3, 6, 3, 16, 32, 2, [(2, list(range(32)))], [(10, 12, 0, 6), (11, 14, 0, 6), (20, 20, 2, 5)], 342),
    "long_window": (1, 2, 1, 128, 4096, 0, [(0, list(range(4096)))], [(0, 4095, 0, 0)], 343),
    "chunk_edges": (1, 4, 2, 128, 1024, 0, [(0, list(range(600)))], [(0, 63, 0, 0), (0, 64, 0, 0), (0, 599, 0, 0)],
                    344),
    "odd_head": (1, 3, 3, 6, 16, 0, [(0, list(range(10)))], [(0, 9, 0, 0), (2, 5, 0, 2)], 345),
    "wide_head": (1, 2, 1, 256, 64, 0, [(0, list(range(50)))], [(0, 49, 0, 0)], 346),
}


@pytest.mark.parametrize("case", list(TOL_CASES))
def test_attention_tolerance_mode(gpu, oracle, case):
    """kernrt_cuda_set_exact(ctx, 0): calls of at most 4 windows take the
    window in chunks of 64 positions summed in parallel and combined; longer
    calls (prefill) stay exact; both within the same bounds."""
    attention_case(gpu, oracle, *TOL_CASES[case], exact=False)


def test_attention_decode_rows_partial_slices_and_ring_wrap(gpu, oracle):
    """Decode-sized calls (few (row, head) pairs): head size 80 (value slices
    of 32, 32 and 16), two query heads per key/value head, windows of 1000 and
    777 positions (the streamed value tiles wrap their ring and end in a
    partial tile), one with a shared range, and a 3-position window."""
    wins = [(0, 999, 0, 0), (300, 1000, 0, 76), (0, 2, 0, 0)]
    attention_case(gpu, oracle, 1, 4, 2, 80, 1024, 0, [(0, list(range(1024)))], wins, 335)


@pytest.mark.parametrize("rows,qw,kvw,head", [(1, 2048, 2048, 64), (5, 1536, 512, 64), (37, 256, 128, 32),
                                            (3, 96, 48, 12)])
def test_rope_then_kv_write_is_one_launch(oracle, rows, qw, kvw, head):
    """The driver's rope(q, k) then kv_write(k, v) (llama.rs:744-757) runs as
    one launch: q and k come out as the oracle's rotation, and the cache holds
    what the separate calls write (a barrier between them keeps them apart):
    attention over either cache gives the same bits."""
    theta, seq, layer = 1.3e5, 64, 1
    q = _data.lcg_normal(rows * qw, 360 + rows).reshape(rows, qw)
    k = _data.lcg_normal(rows * kvw, 361 + rows).reshape(rows, kvw)
    v = _data.lcg_normal(rows * kvw, 362 + rows).reshape(rows, kvw)
    slots = np.array([(7 * r + 3) % seq for r in range(rows)], np.uint64)
    if len(set(slots.tolist())) < rows:
        slots = np.arange(rows, dtype=np.uint64)
    n_heads, kv_mul = qw // head, qw // kvw
    results = {}
    for fused in (True, False):
        with kernrt_b200.CudaBackend(0) as b:
            b.kv_prepare(2, kvw, seq)
            hq, hk, hv = b.upload(q), b.upload(k), b.upload(v)
            b.synchronize()
            n0 = kernrt_b200.kernel_launches()
            b.rope(hq, hk, qw, kvw, rows, slots, head, theta, False)
            if not fused:
                b.synchronize()
            b.kv_write(layer, slots, hk, hv, rows)
            b.synchronize()
            launches = kernrt_b200.kernel_launches() - n0
            got_q, got_k = b.read(hq, rows * qw).reshape(rows, qw), b.read(hk, rows * kvw).reshape(rows, kvw)
            hqa = b.upload(_data.lcg_normal(qw, 363))
            ho, ha = b.alloc(qw), b.alloc(n_heads * seq)
            b.attention(hqa, ho, ha, layer, [(0, seq - 1, 0, 0)], n_heads, kv_mul, head, kvw, seq)
            results[fused] = (launches, got_q, got_k, b.read(ho, qw), b.read(ha, n_heads * seq))
    assert results[True][0] == 1 and results[False][0] == 2
    want_q, want_k = oracle.rope(q, k, slots, head, theta)
    for fused in (True, False):
        assert_bits_equal(results[fused][1], want_q, "rope q")
        assert_bits_equal(results[fused][2], want_k, "rope k")
    assert_bits_equal(results[True][3], results[False][3], "attention over the fused cache")
    assert_bits_equal(results[True][4], results[False][4], "attention weights over the fused cache")


def test_attention_long_window(gpu, oracle):
    attention_case(gpu, oracle, 1, 2, 1, 128, 4096, 0, [(0, list(range(4096)))], [(0, 4095, 0, 0)], 330)


def test_contraction_errors(gpu):
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu.project(12345, gpu.alloc(8), gpu.alloc(8), 1)
    assert "invalid matrix handle" in str(e.value)
    b = kernrt_b200.CudaBackend(0)
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        b.kv_write(0, [0], b.alloc(8), b.alloc(8), 1)
    assert e.value.code == kernrt_b200.E_STATE
    b.kv_prepare(1, 8, 16)
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        b.kv_write(0, [16], b.alloc(8), b.alloc(8), 1)
    assert "out of range" in str(e.value)
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        b.attention(b.alloc(8), b.alloc(8), b.alloc(16), 0, [(5, 3, 0, 0)], 1, 1, 8, 8, 16)
    assert "window 0 out of range" in str(e.value)
    b.synchronize()
    b.close()


def test_attention_odd_head_size(gpu, oracle):
    # head_size 6 takes the single-kernel path
    attention_case(gpu, oracle, 1, 3, 3, 6, 16, 0, [(0, list(range(10)))], [(0, 9, 0, 0), (2, 5, 0, 2)], 340)


@pytest.mark.parametrize("rows", [1, 3, 6])
def test_project_qkv_and_gate_up_equal_the_separate_projections(gpu, oracle, rows):
    """mod.rs:320-337: the fused calls give each projection's own bits, in one
    launch for decode rows, one after another otherwise or when storages differ."""
    dim = 256
    mats = []
    for i, (kind, out) in enumerate([("bf16", 256), ("bf16", 64), ("bf16", 64), ("q8_0", 512), ("q8_0", 512)]):
        dk, data, scales, ok = weights(kind, out, dim, 400 + i, oracle)
        mats.append((gpu.prepare_matrix(dk, data, scales, out, dim), data, scales, ok, out))
    x = _data.lcg_normal(rows * dim, 410 + rows).reshape(rows, dim)
    hx = gpu.upload(x)
    outs = [gpu.alloc(rows * m[4]) for m in mats]
    gpu.synchronize()
    n0 = kernrt_b200.kernel_launches()
    gpu.project_qkv(mats[0][0], mats[1][0], mats[2][0], hx, outs[0], outs[1], outs[2], rows)
    gpu.project_gate_up(mats[3][0], mats[4][0], hx, outs[3], outs[4], rows)
    gpu.synchronize()
    assert kernrt_b200.kernel_launches() - n0 == (2 if rows <= 4 else 5)
    for (h, data, scales, ok, out), ho in zip(mats, outs):
        want = oracle.project(ok, data, scales, out, dim, x)
        assert_bits_equal(gpu.read(ho, rows * out).reshape(rows, out), want, "fused projection")
    # storages that differ take the separate launches, same bits
    dk, data, _, ok = weights("f32", 64, dim, 420, oracle)
    mf = gpu.prepare_matrix(dk, data, None, 64, dim)
    gpu.project_qkv(mats[0][0], mf, mats[2][0], hx, outs[0], outs[1], outs[2], rows)
    assert_bits_equal(gpu.read(outs[1], rows * 64).reshape(rows, 64), oracle.project(ok, data, None, 64, dim, x), "k")
