"""Per-op parity of the CUDA backend against the CPU oracle, through the C ABI.

Every op is bit-exact against the oracle except silu_mul (CUDA expf vs glibc
expf), which is held to |g - r| <= 1e-5 |r|.  Shapes cover the reference
configurations plus ragged/odd sizes that take the kernels' scalar paths.
"""
import numpy as np
import pytest

import kernrt_b200
from tests import _data
from tests._parity import assert_bits_equal, assert_close_rel

pytestmark = pytest.mark.gpu
f32 = np.float32


def up(gpu, a):
    return gpu.upload(np.ascontiguousarray(a, f32))


def rd(gpu, h, shape):
    return gpu.read(h, int(np.prod(shape))).reshape(shape)


# --- embed (reference.rs:133-140) -------------------------------------------------

@pytest.mark.parametrize("vocab,dim", [(64, 96), (49, 576), (97, 2048), (16, 36), (13, 7)])
def test_embed_bf16(gpu, oracle, vocab, dim):
    table = _data.bf16_table(vocab, dim, 1)
    toks = _data.tokens(23, vocab, 2)
    gpu.prepare_embedding(oracle.BF16, table, None, vocab, dim)
    assert gpu.storage() == "bf16"
    out = gpu.alloc(len(toks) * dim)
    for r, t in enumerate(toks):
        gpu.embed(int(t), out, r * dim)
    got = rd(gpu, out, (len(toks), dim))
    assert_bits_equal(got, oracle.embed_rows(oracle.BF16, table, None, vocab, dim, toks), "embed bf16")


@pytest.mark.parametrize("vocab,dim", [(64, 96), (40, 1024), (12, 32)])
def test_embed_q8_0(gpu, oracle, vocab, dim):
    codes, scales = _data.q8_table(vocab, dim, 3)
    toks = _data.tokens(31, vocab, 4)
    gpu.prepare_embedding(oracle.Q8_0, codes, scales, vocab, dim)
    assert gpu.storage() == "q8_0"
    out = gpu.alloc(len(toks) * dim)
    for r, t in enumerate(toks):
        gpu.embed(int(t), out, r * dim)
    got = rd(gpu, out, (len(toks), dim))
    assert_bits_equal(got, oracle.embed_rows(oracle.Q8_0, codes, scales, vocab, dim, toks), "embed q8_0")


def test_embed_q8_0x4_deinterleaves_on_device(gpu, oracle):
    vocab, dim = 32, 128
    w = _data.lcg_normal(vocab * dim, 5, 0.0, 0.05).reshape(vocab, dim)
    blocks = oracle.q8_0x4_pack(w)
    gpu.prepare_embedding(oracle.Q8_0X4, blocks, None, vocab, dim)
    assert gpu.storage() == "q8_0x4"
    toks = _data.tokens(19, vocab, 6)
    out = gpu.alloc(len(toks) * dim)
    for r, t in enumerate(toks):
        gpu.embed(int(t), out, r * dim)
    got = rd(gpu, out, (len(toks), dim))
    assert_bits_equal(got, oracle.embed_rows(oracle.Q8_0X4, blocks, None, vocab, dim, toks), "q8_0x4")


def test_embed_f32_and_unaligned_offsets(gpu, oracle):
    vocab, dim = 20, 12
    table = _data.lcg_normal(vocab * dim, 7).reshape(vocab, dim)
    gpu.prepare_embedding(oracle.F32, table, None, vocab, dim)
    out = gpu.alloc(5 * dim + 3)
    toks = [3, 19, 0, 7, 7]
    for r, t in enumerate(toks):
        gpu.embed(t, out, 3 + r * dim)  # offset 3: scalar path
    got = gpu.read(out, 5 * dim + 3)
    want = np.zeros(5 * dim + 3, f32)
    want[3:] = oracle.embed_rows(oracle.F32, table, None, vocab, dim, toks).ravel()
    assert_bits_equal(got, want, "embed f32")


def test_embed_rejects_bad_token_and_offset(gpu, oracle):
    import kernrt_b200

    table = _data.bf16_table(8, 16, 8)
    gpu.prepare_embedding(oracle.BF16, table, None, 8, 16)
    out = gpu.alloc(32)
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu.embed(8, out, 0)
    assert e.value.code == kernrt_b200.E_INVALID
    with pytest.raises(kernrt_b200.KernrtCudaError):
        gpu.embed(1, out, 17)  # 17 + 16 > 32
    gpu.embed(1, out, 16)  # still usable
    assert_bits_equal(gpu.read(out, 32)[16:], oracle.bf16_to_f32(table[1]), "embed after error")


@pytest.mark.parametrize("kind", ["bf16", "q8_0", "f32"])
@pytest.mark.parametrize("rows", [1, 3, 40])
def test_embed_then_rms_norm_few_rows(gpu, oracle, kind, rows):
    """The driver's embed x rows -> rms_norm pair (llama.rs:734-740) for a few
    rows (decode): one launch, a CTA per row gathering and normalising in the
    reference's order, x keeping the gathered rows; in tolerance mode the
    one-to-four-row form sums the squares by a block reduction."""
    vocab, dim, eps = 300, 1024, 1e-5
    if kind == "bf16":
        table, sc, k = _data.bf16_table(vocab, dim, 60), None, oracle.BF16
    elif kind == "q8_0":
        (table, sc), k = _data.q8_table(vocab, dim, 61), oracle.Q8_0
    else:
        table, sc, k = _data.lcg_normal(vocab * dim, 62).reshape(vocab, dim), None, oracle.F32
    toks = _data.tokens(rows, vocab, 63)
    w = _data.lcg_normal(dim, 64, 1.0, 0.1)
    gpu.prepare_embedding(k, table, sc, vocab, dim)
    hw = gpu.upload(w)
    want_x = oracle.embed_rows(k, table, sc, vocab, dim, toks)
    want = oracle.rms_norm(want_x, w, eps)
    for exact in (True, False):
        x, xb = gpu.alloc(rows * dim), gpu.alloc(rows * dim)
        gpu.set_exact(exact)
        try:
            gpu.synchronize()
            n0 = kernrt_b200.kernel_launches()
            for r, t in enumerate(toks):
                gpu.embed(int(t), x, r * dim)
            gpu.rms_norm(xb, x, hw, rows, dim, eps)
            gpu.synchronize()
            launches = kernrt_b200.kernel_launches() - n0
        finally:
            gpu.set_exact(True)
        assert launches == 1
        assert_bits_equal(rd(gpu, x, (rows, dim)), want_x, f"x ({kind})")
        if exact or rows > 4:
            assert_bits_equal(rd(gpu, xb, (rows, dim)), want, f"xb ({kind})")
        else:
            assert_close_rel(rd(gpu, xb, (rows, dim)), want, rtol=1e-5, what=f"xb ({kind}, block reduction)")


# --- rms_norm (reference.rs:161-178) ---------------------------------------------------

# Enough rows for several row groups per CTA and several column tiles per row
# in the tiled pipeline (2000x8192), rows that wrap each CTA's whole-row ring
# several times (20000x1024, 9001x2048), few rows, and widths that take the
# unaligned fallback.
@pytest.mark.parametrize("rows,dim,eps", [(1, 2048, 1e-5), (7, 576, 1e-5), (33, 1536, 1e-6),
                                          (5, 37, 1e-5), (64, 1024, 1e-6), (3, 8192, 1e-5),
                                          (2, 12, 0.0), (100, 2048, 1e-5), (5000, 2048, 1e-5),
                                          (3001, 576, 1e-6), (2000, 8192, 1e-5), (700, 1000, 1e-5),
                                          (1200, 96, 1e-6), (20000, 1024, 1e-5), (9001, 2048, 1e-6)])
def test_rms_norm(gpu, oracle, rows, dim, eps):
    x = _data.lcg_normal(rows * dim, 10 + dim).reshape(rows, dim)
    w = _data.lcg_normal(dim, 11, 1.0, 0.1)
    hx, hw, ho = up(gpu, x), up(gpu, w), gpu.alloc(rows * dim)
    gpu.rms_norm(ho, hx, hw, rows, dim, eps)
    assert_bits_equal(rd(gpu, ho, (rows, dim)), oracle.rms_norm(x, w, eps), f"rms {rows}x{dim}")


@pytest.mark.parametrize("rows,dim", [(4000, 2048), (300, 1536), (7, 64), (9, 20), (640, 1000), (2000, 64),
                                      (9001, 2048), (5000, 3072)])
def test_add_in_place_then_rms_norm_fuses(gpu, oracle, rows, dim):
    """The driver's add_in_place(x, o) -> rms_norm(xb, x) pair (llama.rs:762-765)
    runs as one launch (for rows of whole float4 pairs) and matches the two ops
    in order."""
    x = _data.lcg_normal(rows * dim, 13 + dim).reshape(rows, dim)
    o = _data.lcg_normal(rows * dim, 14 + dim).reshape(rows, dim)
    w = _data.lcg_normal(dim, 15, 1.0, 0.1)
    hx, ho, hw, hxb = up(gpu, x), up(gpu, o), up(gpu, w), gpu.alloc(rows * dim)
    gpu.synchronize()
    n0 = kernrt_b200.kernel_launches()
    gpu.add_in_place(hx, ho, rows * dim)
    gpu.rms_norm(hxb, hx, hw, rows, dim, 1e-5)
    gpu.synchronize()
    assert kernrt_b200.kernel_launches() - n0 == (1 if dim % 8 == 0 else 2)
    xs = oracle.add_in_place(x, o)
    assert_bits_equal(rd(gpu, hx, (rows, dim)), xs, "x + o")
    assert_bits_equal(rd(gpu, hxb, (rows, dim)), oracle.rms_norm(xs, w, 1e-5), "xb")


@pytest.mark.parametrize("rows,dim", [(1, 2048), (4, 576), (2, 8192), (1, 36), (5, 2048)])
def test_rms_norm_tolerance_mode(gpu, oracle, rows, dim):
    """kernrt_cuda_set_exact(ctx, 0): decode-sized norms (1-4 rows) sum their
    squares by a block reduction (within 1e-5 relative); 5 rows stay exact.
    The add_in_place -> rms_norm pair likewise."""
    x = _data.lcg_normal(rows * dim, 16 + dim).reshape(rows, dim)
    o = _data.lcg_normal(rows * dim, 17 + dim).reshape(rows, dim)
    w = _data.lcg_normal(dim, 18, 1.0, 0.1)
    hx, ho, hw, hxb, hyb = up(gpu, x), up(gpu, o), up(gpu, w), gpu.alloc(rows * dim), gpu.alloc(rows * dim)
    gpu.set_exact(False)
    try:
        gpu.rms_norm(hxb, hx, hw, rows, dim, 1e-5)
        gpu.add_in_place(hx, ho, rows * dim)
        gpu.rms_norm(hyb, hx, hw, rows, dim, 1e-5)
        got, got_add = rd(gpu, hxb, (rows, dim)), rd(gpu, hyb, (rows, dim))
    finally:
        gpu.set_exact(True)
    want = oracle.rms_norm(x, w, 1e-5)
    want_add = oracle.rms_norm(oracle.add_in_place(x, o), w, 1e-5)
    if rows <= 4:
        assert_close_rel(got, want, rtol=1e-5, what="rms_norm (block reduction)")
        assert_close_rel(got_add, want_add, rtol=1e-5, what="add + rms_norm (block reduction)")
    else:
        assert_bits_equal(got, want, "rms_norm, 5 rows")
        assert_bits_equal(got_add, want_add, "add + rms_norm, 5 rows")


def test_rms_norm_partial_rows_leave_the_rest(gpu, oracle):
    rows, dim = 9, 64
    x = _data.lcg_normal(rows * dim, 12).reshape(rows, dim)
    w = np.ones(dim, f32)
    hx, hw, ho = up(gpu, x), up(gpu, w), gpu.alloc(rows * dim)
    gpu.rms_norm(ho, hx, hw, 4, dim, 1e-5)
    got = rd(gpu, ho, (rows, dim))
    assert_bits_equal(got[:4], oracle.rms_norm(x[:4], w, 1e-5), "live rows")
    assert np.all(got[4:] == 0)


def test_rms_norm_rejects_aliasing(gpu):
    import kernrt_b200

    h = gpu.alloc(64)
    w = gpu.alloc(64)
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu.rms_norm(h, h, w, 1, 64, 1e-5)
    assert "distinct" in str(e.value)


# --- qk_norm (reference.rs:180-207) ------------------------------------------------------

@pytest.mark.parametrize("rows,width,head", [(5, 1024, 128), (3, 2048, 64), (2, 1536, 64),
                                             (4, 512, 64), (3, 24, 6), (2, 4096, 64),
                                             (2, 100, 32), (1, 2048, 128), (3000, 2048, 128),
                                             (1200, 1536, 64), (500, 16, 4)])
def test_qk_norm(gpu, oracle, rows, width, head):
    v = _data.lcg_normal(rows * width, 20 + width).reshape(rows, width)
    w = _data.lcg_normal(head, 21, 1.0, 0.1)
    hv, hw = up(gpu, v), up(gpu, w)
    gpu.qk_norm(hv, rows, width, head, hw, 1e-6)
    assert_bits_equal(rd(gpu, hv, (rows, width)), oracle.qk_norm(v, head, w, 1e-6), "qk_norm")


# The driver's qk_norm(q), qk_norm(k), rope(q, k) sequence runs as one launch;
# large row counts give every warp several staged rows, small heads and the
# interleaved form take their own paths.
QK_ROPE_SHAPES = [(3000, 2048, 1024, 128, 1e6), (2500, 1536, 512, 64, 1e6), (7, 2048, 1024, 128, 1e6),
                  (300, 64, 32, 8, 1e4), (40, 8, 8, 4, 1e4), (33, 12, 12, 6, 1e4)]


@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("rows,qw,kvw,head,theta", QK_ROPE_SHAPES)
def test_qk_norm_then_rope_fused(gpu, oracle, rows, qw, kvw, head, theta, interleaved):
    q = _data.lcg_normal(rows * qw, 35 + qw).reshape(rows, qw)
    k = _data.lcg_normal(rows * kvw, 36 + kvw).reshape(rows, kvw)
    wq = _data.lcg_normal(head, 37, 1.0, 0.1)
    wk = _data.lcg_normal(head, 38, 1.0, 0.1)
    pos = (np.arange(rows, dtype=np.uint64) * 7) % 4096
    hq, hk, hwq, hwk = up(gpu, q), up(gpu, k), up(gpu, wq), up(gpu, wk)
    gpu.synchronize()
    n0 = kernrt_b200.kernel_launches()
    gpu.qk_norm(hq, rows, qw, head, hwq, 1e-6)
    gpu.qk_norm(hk, rows, kvw, head, hwk, 1e-6)
    gpu.rope(hq, hk, qw, kvw, rows, pos, head, theta, interleaved)
    gpu.synchronize()
    assert kernrt_b200.kernel_launches() - n0 == 1
    nq, nk = oracle.qk_norm(q, head, wq, 1e-6), oracle.qk_norm(k, head, wk, 1e-6)
    want_q, want_k = oracle.rope(nq, nk, pos, head, theta, interleaved)
    assert_bits_equal(rd(gpu, hq, (rows, qw)), want_q, "q")
    assert_bits_equal(rd(gpu, hk, (rows, kvw)), want_k, "k")


# --- rope (reference.rs:209-257) -----------------------------------------------------------

ROPE_SHAPES = [(6, 576, 192, 64, 1e5), (4, 2048, 2048, 64, 1.3e5), (3, 2048, 1024, 128, 1e6),
               (2, 1536, 512, 64, 1e6), (3, 12, 8, 6, 1e4), (5, 64, 96, 32, 1e4), (2, 8, 8, 4, 1e4)]


@pytest.mark.parametrize("interleaved", [False, True])
@pytest.mark.parametrize("rows,qw,kvw,head,theta", ROPE_SHAPES)
def test_rope(gpu, oracle, rows, qw, kvw, head, theta, interleaved):
    q = _data.lcg_normal(rows * qw, 30 + qw).reshape(rows, qw)
    k = _data.lcg_normal(rows * kvw, 31 + kvw).reshape(rows, kvw)
    pos = np.array([0, 1, 511, 4095, 8191, 3, 77][:rows], np.uint64)
    hq, hk = up(gpu, q), up(gpu, k)
    gpu.rope(hq, hk, qw, kvw, rows, pos, head, theta, interleaved)
    wq, wk = oracle.rope(q, k, pos, head, theta, interleaved)
    assert_bits_equal(rd(gpu, hq, (rows, qw)), wq, "rope q")
    assert_bits_equal(rd(gpu, hk, (rows, kvw)), wk, "rope k")


def test_many_small_staged_slices_wrap_the_staging_ring(oracle):
    """12 000 one-row rope calls with no barrier between them: each stages its
    position (256 bytes of the 1 MB staging ring, read in place by the
    kernel), so the ring wraps three times, every slice ending exactly on a
    segment boundary at some point.  The rotations must come out as the same
    sequence applied by the oracle."""
    head, w = 8, 16
    q = _data.lcg_normal(w, 35).reshape(1, w)
    k = _data.lcg_normal(w, 36).reshape(1, w)
    positions = [int(p) for p in np.random.default_rng(37).integers(0, 64, 12000)]
    with kernrt_b200.CudaBackend(0) as b:  # a fresh ring of the default size
        hq, hk = up(b, q), up(b, k)
        for p in positions:
            b.rope(hq, hk, w, w, 1, [p], head, 1e4, False)
        got_q, got_k = rd(b, hq, (1, w)), rd(b, hk, (1, w))
    wq, wk = q, k
    for p in positions:
        wq, wk = oracle.rope(wq, wk, [p], head, 1e4)
    assert_bits_equal(got_q, wq, "q after 12 000 rotations")
    assert_bits_equal(got_k, wk, "k after 12 000 rotations")


def test_rope_takes_min_of_rows_and_positions(gpu, oracle):
    rows, w, head = 4, 64, 16
    q = _data.lcg_normal(rows * w, 33).reshape(rows, w)
    k = _data.lcg_normal(rows * w, 34).reshape(rows, w)
    hq, hk = up(gpu, q), up(gpu, k)
    gpu.rope(hq, hk, w, w, rows, [5, 9], head, 1e4, False)
    wq, wk = oracle.rope(q[:2], k[:2], [5, 9], head, 1e4)
    got = rd(gpu, hq, (rows, w))
    assert_bits_equal(got[:2], wq, "rope rows")
    assert_bits_equal(got[2:], q[2:], "untouched rows")


# --- silu_mul / add / mul / copy -----------------------------------------------------------

@pytest.mark.parametrize("n", [1, 3, 1000, 1004, 4608, 8192 * 5 + 3])  # 1000, 4608: 256-bit path; 1004: float4
def test_silu_mul(gpu, oracle, n):
    g = _data.lcg_normal(n, 40, 0.0, 3.0)
    u = _data.lcg_normal(n, 41)
    if n > 8:
        g[:8] = [0.0, -0.0, 20.0, -20.0, 80.0, -80.0, 1e-30, -1e-30]
    hg, hu = up(gpu, g), up(gpu, u)
    gpu.silu_mul(hg, hu, n)
    assert_close_rel(gpu.read(hg, n), oracle.silu_mul(g, u), what="silu_mul")


@pytest.mark.parametrize("n", [1, 2, 7, 4096, 65536 + 5])
def test_add_in_place(gpu, oracle, n):
    d = _data.lcg_normal(n, 42)
    s = _data.lcg_normal(n, 43)
    hd, hs = up(gpu, d), up(gpu, s)
    gpu.add_in_place(hd, hs, n)
    assert_bits_equal(gpu.read(hd, n), oracle.add_in_place(d, s), "add")


def test_mul_offsets_and_aliasing(gpu, oracle):
    n = 3 * 1536
    base = _data.lcg_normal(n, 44)
    # the LFM2 pattern: h = B * x over thirds of one buffer into another
    hb = up(gpu, base)
    hh = gpu.alloc(1536)
    gpu.mul(hh, 0, hb, 0, hb, 2 * 1536, 1536)
    want = np.zeros(1536, f32)
    oracle.mul_into(want, 0, base, 0, base, 2 * 1536, 1536)
    assert_bits_equal(gpu.read(hh, 1536), want, "mul thirds")
    # in place, same offsets (benign) and overlapping different offsets (in-order)
    for oo, ao, bo, length in [(0, 0, 100, 500), (10, 0, 2000, 700), (0, 5, 300, 900), (7, 7, 7, 50)]:
        arr = base.copy()
        h = up(gpu, arr)
        gpu.mul(h, oo, h, ao, h, bo, length)
        oracle.mul_into(arr, oo, arr, ao, arr, bo, length)
        assert_bits_equal(gpu.read(h, n), arr, f"mul alias {oo},{ao},{bo}")


def test_copy_overlapping_is_memmove(gpu, oracle):
    n = 1000
    base = _data.lcg_normal(n, 45)
    for so, do, length in [(0, 10, 900), (10, 0, 900), (0, 500, 500), (3, 3, 10)]:
        arr = base.copy()
        h = up(gpu, arr)
        gpu.copy(h, so, h, do, length)
        oracle.copy_into(arr, so, arr, do, length)
        assert_bits_equal(gpu.read(h, n), arr, f"copy {so}->{do}")
    other = gpu.alloc(n)
    h = up(gpu, base)
    gpu.copy(h, 1, other, 0, 2)
    assert list(gpu.read(other, 2)) == list(base[1:3])


# --- conv (reference.rs:365-393, 490-503) -------------------------------------------------

# Row-tiled kernels for k = 2..4 (float4 channels when dim % 4 == 0, tiles of 8
# rows, ragged last tiles, prompts shorter than the halo) and the per-element
# kernel for other sizes.
@pytest.mark.parametrize("rows,dim,k", [(9, 40, 3), (1, 1536, 3), (64, 1536, 3), (5, 8, 1),
                                        (7, 33, 4), (2, 16, 3), (33, 1536, 2), (19, 12, 4),
                                        (1000, 64, 3), (3, 8, 4), (1, 4, 2), (100, 96, 5),
                                        (77, 35, 2)])
def test_conv_prefill(gpu, oracle, rows, dim, k):
    x = _data.lcg_normal(rows * dim, 50 + dim).reshape(rows, dim)
    w = _data.lcg_normal(dim * k, 51, 0.0, 0.3)
    hx, hw, ho = up(gpu, x), up(gpu, w), gpu.alloc(rows * dim)
    gpu.conv_prefill(ho, hx, hw, rows, dim, k)
    assert_bits_equal(rd(gpu, ho, (rows, dim)), oracle.conv_prefill(x, w, k), "conv_prefill")


def test_conv_prefill_in_place_reads_the_original(gpu, oracle):
    rows, dim, k = 6, 16, 3
    x = _data.lcg_normal(rows * dim, 52).reshape(rows, dim)
    w = _data.lcg_normal(dim * k, 53)
    hx, hw = up(gpu, x), up(gpu, w)
    gpu.conv_prefill(hx, hx, hw, rows, dim, k)
    assert_bits_equal(rd(gpu, hx, (rows, dim)), oracle.conv_prefill(x, w, k), "conv in place")


@pytest.mark.parametrize("dim,k", [(4, 3), (1536, 3), (33, 4), (8, 1), (8, 2)])
def test_conv_decode_steps_match_prefill(gpu, oracle, dim, k):
    rows = 6
    h = _data.lcg_normal(rows * dim, 54).reshape(rows, dim)
    w = _data.lcg_normal(dim * k, 55, 0.0, 0.3)
    hw = up(gpu, w)
    state = gpu.alloc(max(1, (k - 1) * dim))
    ost = np.zeros(max(1, (k - 1) * dim), f32)
    for r in range(rows):
        hx = up(gpu, h[r])
        gpu.conv_decode(hx, hx, hw, state, dim, k)  # out aliases x
        want, ost_new = oracle.conv_decode(h[r], w, ost[:(k - 1) * dim] if k > 1 else np.zeros(0, f32), k)
        if k > 1:
            ost[:(k - 1) * dim] = ost_new
        assert_bits_equal(gpu.read(hx, dim), want, f"decode row {r}")
        if k > 1:
            assert_bits_equal(gpu.read(state, (k - 1) * dim), ost[:(k - 1) * dim], f"ring row {r}")


# --- Q8_0 (quant.rs:856-874) -------------------------------------------------------------------

@pytest.mark.parametrize("rows,dim", [(3, 1000), (256, 1024), (2, 37), (1, 2048)])
def test_quantize_q8_0(gpu, oracle, rows, dim):
    x = _data.lcg_normal(rows * dim, 60 + dim).reshape(rows, dim)
    x[0, :5] = [0.0, -0.0, 1e-38, 3.0, -3.0]
    if dim >= 64:
        x[0, 32:64] = 0.0  # an all-zero block: scale 0, inv 0
    nb = (dim + 31) // 32
    hx = up(gpu, x)
    hc, hs, hh = gpu.alloc_bytes(rows * nb * 32), gpu.alloc_bytes(rows * nb * 4), gpu.alloc_bytes(rows * nb * 2)
    gpu.quantize_q8_0(hx, rows, dim, hc, hs, hh)
    wc, ws, wh = oracle.q8_quantize_rows(x)
    assert_bits_equal(gpu.read_bytes(hc, rows * nb * 32, np.int8).reshape(rows, -1), wc, "codes")
    assert_bits_equal(gpu.read_bytes(hs, rows * nb * 4, np.float32).reshape(rows, -1), ws, "scales")
    assert_bits_equal(gpu.read_bytes(hh, rows * nb * 2, np.uint16).reshape(rows, -1), wh, "f16 scales")


@pytest.mark.parametrize("rows,dim,eps", [(256, 1024, 1e-6), (5, 2048, 1e-5), (3, 40, 1e-5),
                                          (5000, 1024, 1e-6), (1000, 4096, 1e-5), (333, 96, 1e-5),
                                          (800, 96, 1e-5), (700, 1536, 1e-6), (20000, 1024, 1e-6),
                                          (1500, 160, 1e-5)])
def test_rms_norm_q8_0_fused(gpu, oracle, rows, dim, eps):
    x = _data.lcg_normal(rows * dim, 70 + dim).reshape(rows, dim)
    w = _data.lcg_normal(dim, 71, 1.0, 0.1)
    nb = (dim + 31) // 32
    hx, hw = up(gpu, x), up(gpu, w)
    hc, hs, hh = gpu.alloc_bytes(rows * nb * 32), gpu.alloc_bytes(rows * nb * 4), gpu.alloc_bytes(rows * nb * 2)
    gpu.rms_norm_q8_0(hx, hw, rows, dim, eps, hc, hs, hh)
    wc, ws, wh = oracle.q8_quantize_rows(oracle.rms_norm(x, w, eps))
    assert_bits_equal(gpu.read_bytes(hc, rows * nb * 32, np.int8).reshape(rows, -1), wc, "codes")
    assert_bits_equal(gpu.read_bytes(hs, rows * nb * 4, np.float32).reshape(rows, -1), ws, "scales")
    assert_bits_equal(gpu.read_bytes(hh, rows * nb * 2, np.uint16).reshape(rows, -1), wh, "f16")


@pytest.mark.parametrize("rows,dim", [(300, 1024), (40, 256)])
def test_quantize_q8_0_edge_blocks(gpu, oracle, rows, dim):
    """The standalone quantiser on the same edge blocks: 1/d overflowing,
    subnormal d, zero blocks, infinities and NaNs."""
    x = _data.lcg_normal(rows * dim, 76 + dim).reshape(rows, dim)
    x[:, 32:64] *= np.float32(1e-41)
    x[:, 64:96] *= np.float32(1e-37)
    x[:, 96:128] = 0.0
    x[:, 128:160] *= np.float32(3e-37)
    x[0, 200] = np.inf
    x[1, 201] = -np.inf
    x[2, 202] = np.nan
    x[3, 224:256] = np.nan
    nb = dim // 32
    hx = up(gpu, x)
    hc, hs, hh = gpu.alloc_bytes(rows * dim), gpu.alloc_bytes(rows * nb * 4), gpu.alloc_bytes(rows * nb * 2)
    gpu.quantize_q8_0(hx, rows, dim, hc, hs, hh)
    with np.errstate(all="ignore"):
        wc, ws, wh = oracle.q8_quantize_rows(x)
    assert (np.abs(wc[:, 32:64]) == 127).any()  # the clamp path ran
    assert_bits_equal(gpu.read_bytes(hc, rows * dim, np.int8).reshape(rows, -1), wc, "codes")
    assert_bits_equal(gpu.read_bytes(hs, rows * nb * 4, np.float32).reshape(rows, -1), ws, "scales")
    assert_bits_equal(gpu.read_bytes(hh, rows * nb * 2, np.uint16).reshape(rows, -1), wh, "f16 scales")


@pytest.mark.parametrize("rows,dim", [(300, 1024), (40, 256)])
def test_rms_norm_q8_0_edge_blocks(gpu, oracle, rows, dim):
    """Blocks at the edges of the Q8_0 arithmetic through the fused kernel:
    amax so small that 1/d overflows (codes +-127 by the clamp), d subnormal
    just above that bound, all-zero blocks, blocks with an infinite product
    (d = inf, inv = 0, codes 0) and a row whose sum overflows (scale 0, NaNs)."""
    eps = 1e-6
    x = _data.lcg_normal(rows * dim, 74 + dim).reshape(rows, dim)
    w = _data.lcg_normal(dim, 75, 1.0, 0.1)
    w[32:64] = 1e-41     # subnormal products: d <= 2^-128, 1/d = inf
    w[64:96] = 1e-37     # amax about 3e-37: d on either side of 2^-128
    w[96:128] = 0.0
    w[128:160] = 3e-37   # d subnormal above 2^-128
    if dim > 160:
        w[160:192] = 3e38  # products past FLT_MAX
    x[1, 7] = np.inf
    x[2, 40] = np.nan
    nb = dim // 32
    hx, hw = up(gpu, x), up(gpu, w)
    hc, hs, hh = gpu.alloc_bytes(rows * dim), gpu.alloc_bytes(rows * nb * 4), gpu.alloc_bytes(rows * nb * 2)
    gpu.rms_norm_q8_0(hx, hw, rows, dim, eps, hc, hs, hh)
    with np.errstate(all="ignore"):
        wc, ws, wh = oracle.q8_quantize_rows(oracle.rms_norm(x, w, eps))
    assert (np.abs(wc[3:, 32:64]) == 127).any()  # the clamp path ran
    assert_bits_equal(gpu.read_bytes(hc, rows * dim, np.int8).reshape(rows, -1), wc, "codes")
    assert_bits_equal(gpu.read_bytes(hs, rows * nb * 4, np.float32).reshape(rows, -1), ws, "scales")
    assert_bits_equal(gpu.read_bytes(hh, rows * nb * 2, np.uint16).reshape(rows, -1), wh, "f16")


def test_embed_many_calls_grow_the_staging_ring(gpu, oracle):
    """300 000 deferred embeds flush as one gather whose ids and offsets
    (3.6 MB) outgrow the initial staging ring: the grown ring must hold them
    and the old one stay valid until the next barrier."""
    vocab, dim, n = 97, 8, 300_000
    table = _data.bf16_table(vocab, dim, 77)
    gpu.prepare_embedding(oracle.BF16, table, None, vocab, dim)
    toks = _data.tokens(n, vocab, 78)
    out = gpu.alloc(n * dim)
    for r, t in enumerate(toks.tolist()):
        gpu.embed(t, out, r * dim)
    got = gpu.read(out, n * dim).reshape(n, dim)
    assert_bits_equal(got, oracle.embed_rows(oracle.BF16, table, None, vocab, dim, toks), "embed x300000")
