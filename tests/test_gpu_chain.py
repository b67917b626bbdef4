"""The fused layer-op chain against the oracle, on every benchmark workload.

Inputs follow the benchmark's distributions: embedding ~N(0, 0.02) in bf16 (or
Q8_0 codes U[-127,127] with scales U(1e-4, 1e-2)), norm weights 1 + N(0, 0.1),
activations N(0, 1).  Everything but the SwiGLU output is compared bit for
bit; SwiGLU is held to 1e-5 relative.
"""
import numpy as np
import pytest

import kernrt_b200
from kernrt_b200 import workloads as W
from tests import _data
from tests._parity import assert_bits_equal, assert_close_rel

pytestmark = pytest.mark.gpu
f32 = np.float32


def make_inputs(wl, seed, rows=None, vocab=None):
    rows = wl.rows if rows is None else rows
    vocab = wl.vocab if vocab is None else vocab
    rng = np.random.default_rng(seed)
    d = {"vocab": vocab}
    if wl.storage == "bf16":
        d["table"] = _data.bf16_table_fast(vocab, wl.dim, seed + 1)
    elif wl.storage == "q8_0":
        d["codes"], d["tscales"] = _data.q8_table_fast(vocab, wl.dim, seed + 1)
    else:
        d["x"] = rng.standard_normal((rows, wl.dim), dtype=f32)
    d["tokens"] = rng.integers(0, vocab, rows, dtype=np.int64).astype(np.int32)
    d["positions"] = wl.positions(0, rows)
    d["w_att"] = (1 + 0.1 * rng.standard_normal(wl.dim)).astype(f32)
    d["q"] = rng.standard_normal((rows, wl.q_dim), dtype=f32)
    d["k"] = rng.standard_normal((rows, wl.kv_dim), dtype=f32)
    d["gate"] = rng.standard_normal((rows, wl.hidden), dtype=f32)
    d["up"] = rng.standard_normal((rows, wl.hidden), dtype=f32)
    d["resid"] = rng.standard_normal((rows, wl.dim), dtype=f32)
    if wl.qk_norm:
        d["w_q"] = (1 + 0.1 * rng.standard_normal(wl.head)).astype(f32)
        d["w_k"] = (1 + 0.1 * rng.standard_normal(wl.head)).astype(f32)
    if wl.final_q8:
        d["w_final"] = (1 + 0.1 * rng.standard_normal(wl.dim)).astype(f32)
    return d


def oracle_chain(oracle, wl, d, interleaved=False):
    kw = dict(dim=wl.dim, q_dim=wl.q_dim, kv_dim=wl.kv_dim, hidden=wl.hidden, head=wl.head,
              eps=wl.eps, theta=wl.theta, positions=d["positions"].astype(np.uint64),
              w_att=d["w_att"], q=d["q"], k=d["k"], gate=d["gate"], up=d["up"], resid=d["resid"],
              interleaved=interleaved, w_q=d.get("w_q"), w_k=d.get("w_k"), w_final=d.get("w_final"),
              threads=8)
    if wl.storage == "bf16":
        kw.update(tokens=d["tokens"], table=(oracle.BF16, d["table"], None, d["vocab"]))
    elif wl.storage == "q8_0":
        kw.update(tokens=d["tokens"], table=(oracle.Q8_0, d["codes"], d["tscales"], d["vocab"]))
    else:
        kw.update(x=d["x"])
    return oracle.chain(**kw)


def gpu_chain(gpu, wl, d, interleaved=False):
    rows = d["tokens"].size
    if wl.storage == "bf16":
        gpu.prepare_embedding(kernrt_b200.BF16, d["table"], None, d["vocab"], wl.dim)
    elif wl.storage == "q8_0":
        gpu.prepare_embedding(kernrt_b200.Q8_0, d["codes"], d["tscales"], d["vocab"], wl.dim)
    h = {}
    h["x"] = gpu.upload(d["x"]) if "x" in d else gpu.alloc(rows * wl.dim)
    for n in ["w_att", "q", "k", "gate", "up", "resid", "w_q", "w_k", "w_final"]:
        if n in d:
            h[n] = gpu.upload(d[n])
    h["xb"] = gpu.alloc(rows * wl.dim)
    h["tokens"] = gpu.upload_bytes(d["tokens"])
    h["positions"] = gpu.upload_bytes(d["positions"])
    nb = (wl.dim + 31) // 32
    if wl.final_q8:
        h["codes"] = gpu.alloc_bytes(rows * nb * 32)
        h["scales"] = gpu.alloc_bytes(rows * nb * 4)
        h["scales_f16"] = gpu.alloc_bytes(rows * nb * 2)
    gpu.rope_prepare(wl.theta, wl.head, int(d["positions"].max()) + 1)
    gpu.layer_chain(rows=rows, dim=wl.dim, q_dim=wl.q_dim, kv_dim=wl.kv_dim, hidden=wl.hidden,
                    head_size=wl.head, eps=wl.eps, theta=wl.theta, final_eps=wl.eps,
                    interleaved=int(interleaved),
                    tokens=h["tokens"] if wl.storage != "none" else 0, positions=h["positions"],
                    x=h["x"], xb=h["xb"], w_att=h["w_att"], q=h["q"], k=h["k"], w_q=h.get("w_q", 0),
                    w_k=h.get("w_k", 0), gate=h["gate"], up=h["up"], resid=h["resid"],
                    w_final=h.get("w_final", 0), codes=h.get("codes", 0), scales=h.get("scales", 0),
                    scales_f16=h.get("scales_f16", 0))
    out = {
        "x": gpu.read(h["x"], rows * wl.dim).reshape(rows, wl.dim),
        "xb": gpu.read(h["xb"], rows * wl.dim).reshape(rows, wl.dim),
        "q": gpu.read(h["q"], rows * wl.q_dim).reshape(rows, wl.q_dim),
        "k": gpu.read(h["k"], rows * wl.kv_dim).reshape(rows, wl.kv_dim),
        "gate": gpu.read(h["gate"], rows * wl.hidden).reshape(rows, wl.hidden),
    }
    if wl.final_q8:
        out["codes"] = gpu.read_bytes(h["codes"], rows * nb * 32, np.int8).reshape(rows, -1)
        out["scales"] = gpu.read_bytes(h["scales"], rows * nb * 4, np.float32).reshape(rows, -1)
        out["scales_f16"] = gpu.read_bytes(h["scales_f16"], rows * nb * 2, np.uint16).reshape(rows, -1)
    return out


def check(got, want, final_q8):
    for n in ["x", "xb", "q", "k"]:
        assert_bits_equal(got[n], want[n], n)
    assert_close_rel(got["gate"], want["gate"], what="gate (SwiGLU)")
    if final_q8:
        for n in ["codes", "scales", "scales_f16"]:
            assert_bits_equal(got[n], want[n], n)


@pytest.mark.parametrize("wl", [W.SMOLLM2_135M, W.SMOLLM2_17B_DECODE, W.SMOLLM2_17B_PREFILL,
                                W.QWEN3_06B_Q8], ids=lambda w: w.name)
def test_chain_matches_oracle(gpu, oracle, wl):
    d = make_inputs(wl, 1000)
    check(gpu_chain(gpu, wl, d), oracle_chain(oracle, wl, d), wl.final_q8)


@pytest.mark.parametrize("rows", [8192, 5000, 149, 37])
def test_chain_few_rows_per_sm(gpu, oracle, rows):
    """A shard's row count on 8 GPUs (8 192) and ragged counts: the row-scale
    pass with its last CTA partly filled, and fewer rows than SMs."""
    wl = W.SMOLLM2_17B_PREFILL
    d = make_inputs(wl, 1010 + rows, rows=rows, vocab=4096)
    check(gpu_chain(gpu, wl, d), oracle_chain(oracle, wl, d), False)


def test_chain_few_rows_bad_token_reports_and_recovers(gpu, oracle):
    wl = W.Workload("small", 512, 64, 2, 2, 32, 64, 1e4, 1e-5, "bf16", rows=300, seq_len=300)
    d = make_inputs(wl, 1011)
    d["tokens"][171] = 512  # one past the vocabulary
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu_chain(gpu, wl, d)
    assert e.value.code == kernrt_b200.E_DEVICE
    assert "token id out of range" in str(e.value)
    d["tokens"][171] = 511
    check(gpu_chain(gpu, wl, d), oracle_chain(oracle, wl, d), False)


def test_chain_interleaved_rope(gpu, oracle):
    wl = W.SMOLLM2_135M
    d = make_inputs(wl, 1001, vocab=512)
    check(gpu_chain(gpu, wl, d, interleaved=True), oracle_chain(oracle, wl, d, interleaved=True), False)


def test_chain_lfm2_attention_block(gpu, oracle):
    """LFM2 attention layers: x is an input (no embed), q/k norms, RoPE 1e6."""
    wl = W.LFM2_700M
    d = make_inputs(wl, 1002)
    check(gpu_chain(gpu, wl, d), oracle_chain(oracle, wl, d), False)


@pytest.mark.parametrize("rows,dim,q,kv,head,hidden", [(37, 40, 48, 16, 8, 20), (3, 36, 12, 12, 6, 7),
                                                       (70, 96, 96, 32, 32, 64), (21, 40, 12, 8, 4, 20)])
def test_chain_ragged_shapes(gpu, oracle, rows, dim, q, kv, head, hidden):
    wl = W.Workload("ragged", 50, dim, q // head, kv // head, head, hidden, 1e4, 1e-5, "bf16",
                    rows=rows, seq_len=17, qk_norm=True, final_q8=True)
    d = make_inputs(wl, 1003)
    check(gpu_chain(gpu, wl, d), oracle_chain(oracle, wl, d), True)


@pytest.mark.parametrize("rows,dim", [(300, 1024), (5, 96), (1000, 2048), (170, 544)])
def test_chain_x_input_with_final_q8(gpu, oracle, rows, dim):
    """An x input (no embed) with the final RMSNorm + Q8_0 and a residual: the
    f32 norm stage sums x and x + resid and writes xb, x + resid and the codes
    (the column-tiled pipeline, or a CTA per row for a few rows)."""
    wl = W.Workload("x_fq", 64, dim, 4, 2, 16, 64, 1e4, 1e-6, "none", rows=rows, seq_len=64, qk_norm=False,
                    final_q8=True)
    d = make_inputs(wl, 1010 + rows)
    check(gpu_chain(gpu, wl, d), oracle_chain(oracle, wl, d), True)


def test_chain_bad_token_reports_and_recovers(gpu, oracle):
    wl = W.Workload("tiny", 16, 64, 2, 2, 32, 64, 1e4, 1e-5, "bf16", rows=8, seq_len=8)
    d = make_inputs(wl, 1004)
    d["tokens"][3] = 16  # one past the vocabulary
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu_chain(gpu, wl, d)
    assert e.value.code == kernrt_b200.E_DEVICE
    assert "token id out of range" in str(e.value)
    d["tokens"][3] = 15
    check(gpu_chain(gpu, wl, d), oracle_chain(oracle, wl, d), False)


def test_chain_position_outside_table_reports(gpu):
    wl = W.Workload("tiny", 16, 64, 2, 2, 32, 64, 1e4, 1e-5, "bf16", rows=4, seq_len=4)
    d = make_inputs(wl, 1005)
    gpu.prepare_embedding(kernrt_b200.BF16, d["table"], None, 16, 64)
    h = {n: gpu.upload(d[n]) for n in ["w_att", "q", "k", "gate", "up", "resid"]}
    x, xb = gpu.alloc(4 * 64), gpu.alloc(4 * 64)
    pos = gpu.upload_bytes(np.array([0, 1, 2, 10 ** 6], np.int32))
    gpu.rope_prepare(7777.0, 32, 16)
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu.layer_chain(rows=4, dim=64, q_dim=64, kv_dim=64, hidden=64, head_size=32, eps=1e-5,
                        theta=7777.0, tokens=gpu.upload_bytes(d["tokens"]), positions=pos, x=x, xb=xb,
                        **h)
        gpu.synchronize()
    assert "RoPE table" in str(e.value)
    gpu.synchronize()  # the context stays usable


@pytest.mark.parametrize("rows,dim,k", [(1024, 1536, 3), (37, 100, 2), (13, 33, 4), (9, 64, 5),
                                        (3, 8, 4), (4, 12, 3), (6, 7, 2)])
def test_lfm2_conv_block(gpu, oracle, rows, dim, k):
    rng = np.random.default_rng(7 + rows + k)
    bcx = rng.standard_normal((rows, 3 * dim), dtype=f32)
    kernel = (0.3 * rng.standard_normal(dim * k)).astype(f32)
    ring0 = rng.standard_normal((k - 1) * dim, dtype=f32)
    hb, hk, hr, hc = gpu.upload(bcx), gpu.upload(kernel), gpu.upload(ring0), gpu.alloc(rows * dim)
    gpu.lfm2_conv_block(hb, hk, hr, hc, rows, dim, k)
    cy, ring = oracle.lfm2_conv_block(bcx, kernel, ring0, k)
    assert_bits_equal(gpu.read(hc, rows * dim).reshape(rows, dim), cy, "cy")
    assert_bits_equal(gpu.read(hr, (k - 1) * dim), ring, "ring")


@pytest.mark.parametrize("rows", [1, 2, 5])
def test_lfm2_conv_block_short_prompt_ring(gpu, oracle, rows):
    dim, k = 64, 3
    rng = np.random.default_rng(rows)
    bcx = rng.standard_normal((rows, 3 * dim), dtype=f32)
    kernel = rng.standard_normal(dim * k).astype(f32)
    ring0 = rng.standard_normal((k - 1) * dim, dtype=f32)
    hb, hk, hr, hc = gpu.upload(bcx), gpu.upload(kernel), gpu.upload(ring0), gpu.alloc(rows * dim)
    gpu.lfm2_conv_block(hb, hk, hr, hc, rows, dim, k)
    cy, ring = oracle.lfm2_conv_block(bcx, kernel, ring0, k)
    assert_bits_equal(gpu.read(hc, rows * dim).reshape(rows, dim), cy, "cy")
    assert_bits_equal(gpu.read(hr, (k - 1) * dim), ring, "ring")


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("seq_lens,dim,k", [([1024], 1536, 3), ([100, 50, 200], 48, 3), ([9, 40], 64, 4),
                                            ([30], 12, 2), ([64], 7, 5)])
def test_lfm2_conv_block_sharded_with_halo(gpu, oracle, world, seq_lens, dim, k):
    """kernrt_cuda_lfm2_conv_block_halo: the sequences cut into the row blocks
    of `world` ranks (W.conv_shards), each segment run from its own rows and
    its staged halo (the k - 1 rows of the sequence before it), emulated one
    rank after another on one device: the segments reassemble the unsharded
    block bit for bit, and the segment that ends each sequence seeds its ring."""
    rng = np.random.default_rng(sum(seq_lens) + dim + k)
    bcx = [rng.standard_normal((n, 3 * dim), dtype=f32) for n in seq_lens]
    kernel = (0.3 * rng.standard_normal(dim * k)).astype(f32)
    hk = gpu.upload(kernel)
    full = [oracle.lfm2_conv_block(b, kernel, np.zeros((k - 1) * dim, f32), k) for b in bcx]
    covered = [np.zeros(n, bool) for n in seq_lens]
    for rank in range(world):
        for seq, lo, hi, halo, ends in W.conv_shards(seq_lens, world, rank, k):
            n = hi - lo
            hb, hc = gpu.upload(bcx[seq][lo - halo:hi]), gpu.alloc(n * dim)
            hr = gpu.alloc((k - 1) * dim) if ends and (halo == 0 or n >= k - 1) else 0
            gpu.lfm2_conv_block_halo(hb, hk, hr, hc, n, dim, k, halo)
            assert_bits_equal(gpu.read(hc, n * dim).reshape(n, dim), full[seq][0][lo:hi],
                              f"world {world} rank {rank}: sequence {seq} rows {lo}:{hi}")
            if hr:
                assert_bits_equal(gpu.read(hr, (k - 1) * dim), full[seq][1], f"ring of sequence {seq}")
            covered[seq][lo:hi] = True
    assert all(c.all() for c in covered)


def test_lfm2_conv_block_halo_rejects_what_it_cannot_do(gpu):
    dim, k = 16, 3
    hb, hk, hr, hc = gpu.upload(np.zeros((4, 3 * dim), f32)), gpu.upload(np.zeros(dim * k, f32)), \
        gpu.alloc((k - 1) * dim), gpu.alloc(4 * dim)
    for args, words in [((hb, hk, hr, hc, 2, dim, k, 3), "halo"), ((hb, hk, hr, hc, 1, dim, k, 2), "k - 1 rows"),
                        ((hb, hk, hr, hc, 4, dim, k, 1), "conv block bcx")]:
        with pytest.raises(kernrt_b200.KernrtCudaError) as e:
            gpu.lfm2_conv_block_halo(*args)
        assert e.value.code == kernrt_b200.E_INVALID and words in str(e.value), str(e.value)
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu.lfm2_conv_block(hb, hk, 0, hc, 4, dim, k)
    assert "ring" in str(e.value)


def test_lfm2_conv_block_matches_the_unfused_ops(gpu):
    """The fused block equals the driver's own op sequence (lfm2.rs:584-624)
    run through the backend's trait ops."""
    rows, dim, k = 33, 48, 3
    rng = np.random.default_rng(9)
    bcx = rng.standard_normal((rows, 3 * dim), dtype=f32)
    kernel = rng.standard_normal(dim * k).astype(f32)
    hb, hk = gpu.upload(bcx), gpu.upload(kernel)
    ring_a, cy_a = gpu.alloc((k - 1) * dim), gpu.alloc(rows * dim)
    gpu.lfm2_conv_block(hb, hk, ring_a, cy_a, rows, dim, k)
    h, co, cy, ring = gpu.alloc(rows * dim), gpu.alloc(rows * dim), gpu.alloc(rows * dim), gpu.alloc((k - 1) * dim)
    for r in range(rows):
        gpu.mul(h, r * dim, hb, r * 3 * dim, hb, r * 3 * dim + 2 * dim, dim)
    gpu.conv_prefill(co, h, hk, rows, dim, k)
    take = min(rows, k - 1)
    gpu.copy(h, (rows - take) * dim, ring, (k - 1 - take) * dim, take * dim)
    for r in range(rows):
        gpu.mul(cy, r * dim, hb, r * 3 * dim + dim, co, r * dim, dim)
    assert_bits_equal(gpu.read(cy_a, rows * dim), gpu.read(cy, rows * dim), "cy")
    assert_bits_equal(gpu.read(ring_a, (k - 1) * dim), gpu.read(ring, (k - 1) * dim), "ring")


def test_headline_workload_full_size_sampled(gpu, oracle):
    """65536 rows through the SmolLM2-1.7B chain at full vocabulary: inputs
    generated on the device, 1024 sampled rows (every CTA-boundary row among
    them) compared bit for bit with the oracle."""
    import torch

    from kernrt_b200.interop import as_torch

    wl = W.SMOLLM2_17B_65K
    R, H, Q, KV, I = wl.rows, wl.dim, wl.q_dim, wl.kv_dim, wl.hidden
    table = _data.bf16_table_fast(wl.vocab, H, 42)
    gpu.prepare_embedding(kernrt_b200.BF16, table, None, wl.vocab, H)
    rng = np.random.default_rng(43)
    w_att = (1 + 0.1 * rng.standard_normal(H)).astype(f32)
    tokens = rng.integers(0, wl.vocab, R).astype(np.int32)
    positions = wl.positions()
    h = {n: gpu.alloc(R * w) for n, w in [("x", H), ("xb", H), ("q", Q), ("k", KV), ("gate", I),
                                           ("up", I), ("resid", H)]}
    g = torch.Generator(device="cuda:0").manual_seed(44)
    for n, w in [("q", Q), ("k", KV), ("gate", I), ("up", I), ("resid", H)]:
        as_torch(gpu, h[n], (R, w)).copy_(torch.randn(R, w, device="cuda:0", generator=g))
    torch.cuda.synchronize()
    sample = np.unique(np.concatenate([np.arange(0, R, 16), [R - 1]]))
    sample = np.unique(np.concatenate([rng.choice(sample, 1000, replace=False), [0, 15, 16, R - 1]]))
    ts = torch.as_tensor(sample, device="cuda:0")
    before = {n: as_torch(gpu, h[n], (R, w))[ts].cpu().numpy()
              for n, w in [("q", Q), ("k", KV), ("gate", I), ("up", I), ("resid", H)]}
    gpu.rope_prepare(wl.theta, wl.head, wl.seq_len)
    gpu.layer_chain(rows=R, dim=H, q_dim=Q, kv_dim=KV, hidden=I, head_size=wl.head, eps=wl.eps,
                    theta=wl.theta, tokens=gpu.upload_bytes(tokens),
                    positions=gpu.upload_bytes(positions), x=h["x"], xb=h["xb"],
                    w_att=gpu.upload(w_att), q=h["q"], k=h["k"], gate=h["gate"], up=h["up"],
                    resid=h["resid"])
    gpu.synchronize()
    after = {n: as_torch(gpu, h[n], (R, w))[ts].cpu().numpy()
             for n, w in [("x", H), ("xb", H), ("q", Q), ("k", KV), ("gate", I)]}
    want = oracle.chain(dim=H, q_dim=Q, kv_dim=KV, hidden=I, head=wl.head, eps=wl.eps, theta=wl.theta,
                        positions=positions[sample].astype(np.uint64), w_att=w_att, q=before["q"],
                        k=before["k"], gate=before["gate"], up=before["up"], resid=before["resid"],
                        tokens=tokens[sample], table=(oracle.BF16, table, None, wl.vocab), threads=8)
    check(after, want, False)


def test_stage_timing_records_each_kernel(gpu):
    """kernrt_cuda_stage_timing/_stage_times: the Llama chain issues the norm
    pipeline and the RoPE/SwiGLU stream; each is timed once per launch."""
    wl = W.Workload("tiny", 64, 256, 4, 4, 64, 512, 1e4, 1e-5, "bf16", rows=300, seq_len=300)
    d = make_inputs(wl, 1006)
    gpu.stage_timing(True)
    gpu_chain(gpu, wl, d)
    gpu_chain(gpu, wl, d)
    t = gpu.stage_times()
    gpu.stage_timing(False)
    assert t["norm"][1] == 2 and t["stream"][1] == 2 and t["fused"][1] == 0
    assert t["norm"][0] > 0 and t["stream"][0] > 0


@pytest.mark.parametrize("wl,chunk", [(W.SMOLLM2_135M, 37), (W.QWEN3_06B_Q8, 0), (W.LFM2_700M, 100),
                                      (W.SMOLLM2_17B_PREFILL, 64)], ids=lambda v: str(getattr(v, "name", v)))
def test_chain_on_host_buffers_matches_oracle(gpu, oracle, wl, chunk):
    """kernrt_cuda_layer_chain_host: the same chain on host arrays, pipelined in
    row chunks (outputs written over their inputs here, which is allowed)."""
    d = make_inputs(wl, 1010)
    rows, nb = wl.rows, (wl.dim + 31) // 32
    if wl.storage == "bf16":
        gpu.prepare_embedding(kernrt_b200.BF16, d["table"], None, d["vocab"], wl.dim)
    elif wl.storage == "q8_0":
        gpu.prepare_embedding(kernrt_b200.Q8_0, d["codes"], d["tscales"], d["vocab"], wl.dim)
    w = {n: gpu.upload(d[n]) for n in ["w_att", "w_q", "w_k", "w_final"] if n in d}
    q, k, gate = d["q"].copy(), d["k"].copy(), d["gate"].copy()
    x_out = np.zeros((rows, wl.dim), f32)
    xb_out = np.zeros((rows, wl.dim), f32)
    codes = np.zeros((rows, nb * 32), np.int8) if wl.final_q8 else None
    scales = np.zeros((rows, nb), f32) if wl.final_q8 else None
    s16 = np.zeros((rows, nb), np.uint16) if wl.final_q8 else None
    gpu.layer_chain_host(rows=rows, dim=wl.dim, q_dim=wl.q_dim, kv_dim=wl.kv_dim, hidden=wl.hidden,
                         head_size=wl.head, eps=wl.eps, theta=wl.theta, final_eps=wl.eps, chunk_rows=chunk,
                         tokens=d["tokens"] if wl.storage != "none" else None,
                         positions=d["positions"], x_in=d.get("x"), q_in=q, k_in=k, gate_in=gate,
                         up=d["up"], resid=d["resid"], x_out=x_out, xb_out=xb_out, q_out=q, k_out=k,
                         gate_out=gate, codes=codes, scales=scales, scales_f16=s16, **w)
    got = {"x": x_out, "xb": xb_out, "q": q, "k": k, "gate": gate, "codes": codes, "scales": scales,
           "scales_f16": s16}
    check(got, oracle_chain(oracle, wl, d), wl.final_q8)


def test_chain_on_host_buffers_rejects_bad_token(gpu):
    wl = W.Workload("tiny", 16, 64, 2, 2, 32, 64, 1e4, 1e-5, "bf16", rows=8, seq_len=8)
    d = make_inputs(wl, 1011)
    gpu.prepare_embedding(kernrt_b200.BF16, d["table"], None, 16, 64)
    d["tokens"][5] = -1
    out = np.zeros((8, 64), f32)
    with pytest.raises(kernrt_b200.KernrtCudaError) as e:
        gpu.layer_chain_host(rows=8, dim=64, eps=1e-5, tokens=d["tokens"], x_out=out,
                             w_att=gpu.upload(d["w_att"]))
    assert e.value.code == kernrt_b200.E_INVALID and "out of range" in str(e.value)
