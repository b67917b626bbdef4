"""Per-op and per-workload throughput of the backend (1 GPU).

    python -m kernrt_b200.opbench [--reps N] [--json] [--only REGEX]

Times every row op of the trait, the fused driver pairs, the fused chain on
each benchmark workload and the single-row decode latency, with CUDA events on
the backend's stream (inputs resident in HBM; working sets far above the
126 MB L2 except where a row says otherwise).  GB/s is compulsory bytes over
time; the fraction is against the measured copy bandwidth in
MEASURED_PEAKS.json when present.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import time

import numpy as np

from . import BF16, Q8_0, CudaBackend, kernel_launches
from . import workloads as W
from .interop import as_torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def peak_gbs():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["hbm_gbs"])
    except Exception:
        return 6650.0


class Bench:
    def __init__(self, reps: int, only: str | None = None):
        import torch

        self.torch = torch
        self.b = CudaBackend(0)
        self.stream = torch.cuda.ExternalStream(self.b.stream(), device="cuda:0")
        self.g = torch.Generator(device="cuda:0").manual_seed(0)
        self.reps = reps
        self.only = re.compile(only) if only else None
        self.peak = peak_gbs()
        self.rows = []

    def want(self, *names):
        """Whether any op named by these (sub)strings passes --only."""
        if self.only is None:
            return True
        return any(self.only.search(n) or n in self.only.pattern for n in names)

    def fill(self, h, n, scale=1.0):
        self.b.synchronize()
        as_torch(self.b, h, (n,)).copy_(torch_randn(self, n) * scale)
        self.torch.cuda.synchronize()

    def buf(self, n, scale=1.0):
        h = self.b.alloc(n)
        self.fill(h, n, scale)
        return h

    def time(self, name, fn, nbytes, setup=None, note=""):
        """Median device time per call.  Without a setup step the calls run back
        to back between one pair of events, so host-side work per call (e.g.
        staging host positions) overlaps the previous call's kernels; with one
        (a device copy restoring an in-place input), each call is timed alone
        and its host work overlaps that copy."""
        torch = self.torch
        if self.only is not None and not self.only.search(name):
            return None
        for _ in range(3):
            if setup:
                setup()
            fn()
        self.b.synchronize()
        n0 = kernel_launches()
        times = []
        if setup is None:
            for _ in range(3):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(self.stream)
                for _ in range(self.reps):
                    fn()
                self.b.flush()
                e.record(self.stream)
                e.synchronize()
                times.append(s.elapsed_time(e) / self.reps)
            calls = 3 * self.reps
        else:
            for _ in range(self.reps):
                setup()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(self.stream)
                fn()
                self.b.flush()  # launch any op the backend holds for fusion
                e.record(self.stream)
                e.synchronize()
                times.append(s.elapsed_time(e))
            calls = self.reps
        launches = (kernel_launches() - n0) / calls
        ms = statistics.median(times)
        gbs = nbytes / (ms / 1e3) / 1e9 if nbytes else None
        row = {"name": name, "ms": ms, "ms_min": min(times), "gbs": gbs,
               "frac": None if gbs is None else gbs / self.peak, "launches": launches, "note": note}
        self.rows.append(row)
        return row


def torch_randn(bench, n):
    return bench.torch.randn(n, device="cuda:0", generator=bench.g)


def run(reps: int, only: str | None = None):
    import torch

    B = Bench(reps, only)
    b = B.b
    wl = W.SMOLLM2_17B_65K
    R, H, Q, KV, I = wl.rows, wl.dim, wl.q_dim, wl.kv_dim, wl.hidden
    positions = wl.positions()

    # --- a1 embed, a2 rms_norm and the fused driver pairs (SmolLM2-1.7B rows)
    if B.want("embed", "rms_norm 65536x2048", "add_in_place"):
        table = (torch.randn(wl.vocab, H, device="cuda:0", generator=B.g) * 0.02).to(torch.bfloat16)
        b.prepare_embedding(BF16, table.view(torch.int16).cpu().numpy().view(np.uint16), None, wl.vocab, H)
        del table
        w = b.upload(np.ones(H, np.float32))
        tokens = np.random.default_rng(1).integers(0, wl.vocab, R).astype(np.int32)
        x, xb = b.alloc(R * H), b.alloc(R * H)

        def embed_all():
            for r in range(R):
                b.embed(int(tokens[r]), x, r * H)

        B.time("embed (65536 per-row calls, bf16 table)", embed_all, R * (2 * H + 4 * H),
               note="host loop of 65536 calls included")
        B.fill(x, R * H)
        B.time("rms_norm 65536x2048", lambda: b.rms_norm(xb, x, w, R, H, 1e-5), R * 8 * H)
        o = B.buf(R * H)
        x0 = B.buf(R * H)

        def add_rms():
            b.add_in_place(x, o, R * H)
            b.rms_norm(xb, x, w, R, H, 1e-5)

        B.time("add_in_place + rms_norm (fused)", add_rms, R * 16 * H, setup=lambda: b.copy(x0, 0, x, 0, R * H))
        B.time("add_in_place 65536x2048", lambda: b.add_in_place(x, o, R * H), R * 12 * H,
               setup=lambda: b.copy(x0, 0, x, 0, R * H))

        def embed_rms():
            embed_all()
            b.rms_norm(xb, x, w, R, H, 1e-5)

        B.time("embed x65536 + rms_norm (fused)", embed_rms, R * (2 * H + 8 * H),
               note="host loop of 65536 calls included")

    # --- a3/a4 qk_norm, rope and the fused triple (Qwen3 shape: 16x128 / 8x128)
    if B.want("qk_norm", "rope"):
        qd, kd, hd = 2048, 1024, 128
        q, k = B.buf(R * qd), B.buf(R * kd)
        wq = b.upload(np.ones(hd, np.float32))
        B.time("qk_norm q 65536x(16x128)", lambda: b.qk_norm(q, R, qd, hd, wq, 1e-6), R * 8 * qd)
        B.time("rope q,k 65536x(16+8)x128", lambda: b.rope(q, k, qd, kd, R, positions, hd, 1e6, False),
               R * 8 * (qd + kd))

        def qk_rope():
            b.qk_norm(q, R, qd, hd, wq, 1e-6)
            b.qk_norm(k, R, kd, hd, wq, 1e-6)
            b.rope(q, k, qd, kd, R, positions, hd, 1e6, False)

        B.time("qk_norm q + qk_norm k + rope (fused)", qk_rope, R * 8 * (qd + kd))

    # --- a5 silu_mul
    if B.want("silu_mul"):
        g, u = B.buf(R * I), B.buf(R * I)
        g0 = b.alloc(R * I)
        b.copy(g, 0, g0, 0, R * I)
        B.time("silu_mul 65536x8192", lambda: b.silu_mul(g, u, R * I), R * 12 * I,
               setup=lambda: b.copy(g0, 0, g, 0, R * I))

    # --- a7/a8 LFM2 conv (1024 rows x 1536, and 16384 rows for bandwidth)
    for rows in (1024, 16384):
        if not B.want(f"{rows}x1536"):
            continue
        d = 1536
        bcx, kern = B.buf(rows * 3 * d), B.buf(d * 3, 0.3)
        h, co, cy, ring = b.alloc(rows * d), b.alloc(rows * d), b.alloc(rows * d), b.alloc(2 * d)
        B.time(f"mul (B*x) {rows}x1536", lambda: [b.mul(h, r * d, bcx, r * 3 * d, bcx, r * 3 * d + 2 * d, d)
                                                   for r in range(rows)], rows * 12 * d,
               note="per-row calls (host loop included), batched into one launch")
        B.time(f"conv_prefill {rows}x1536 k3", lambda: b.conv_prefill(co, h, kern, rows, d, 3), rows * 8 * d)
        B.time(f"lfm2_conv_block {rows}x1536 (fused)", lambda: b.lfm2_conv_block(bcx, kern, ring, cy, rows, d, 3),
               rows * 16 * d)

    # --- a9 conv_decode latency, a11 Q8
    d = 1536
    if B.want("conv_decode"):
        xr, kern, st = B.buf(d), B.buf(d * 3), B.buf(2 * d)
        B.time("conv_decode 1x1536 (latency)", lambda: b.conv_decode(xr, xr, kern, st, d, 3), None)
    if B.want("quantize_q8_0", "rms_norm_q8_0"):
        qd8 = 1024
        xq = B.buf(R * qd8)
        nb = qd8 // 32
        c8, s8, h8 = b.alloc_bytes(R * qd8), b.alloc_bytes(R * nb * 4), b.alloc_bytes(R * nb * 2)
        wq8 = b.upload(np.ones(qd8, np.float32))
        B.time("quantize_q8_0 65536x1024", lambda: b.quantize_q8_0(xq, R, qd8, c8, s8, h8),
               R * (4 * qd8 + qd8 + 6 * nb))
        B.time("rms_norm_q8_0 65536x1024 (fused)", lambda: b.rms_norm_q8_0(xq, wq8, R, qd8, 1e-6, c8, s8, h8),
               R * (4 * qd8 + qd8 + 6 * nb))

    # --- contractions (exact order; SmolLM2-1.7B and Qwen3-0.6B shapes)
    if B.want("project", "logits", "attention", "kv_write"):
        contractions(B)

    # --- loading the token embedding from a safetensors file (hf.rs:141-191)
    if B.want("prepare_embedding_file"):
        load_table(B)

    # --- the chain on every workload
    for wk in (W.SMOLLM2_135M, W.SMOLLM2_17B_PREFILL, W.QWEN3_06B_Q8, W.LFM2_700M, W.SMOLLM2_17B_65K):
        if B.want(f"chain: {wk.name}"):
            chain_time(B, wk)

    # --- decode latency: one row through the trait ops, read() each step
    if B.want("decode step"):
        decode_latency(B)
    if B.want("decode token"):
        model_decode(B)
    # --- LFM2-700M's whole layer stack of row ops
    if B.want("lfm2 layer stack"):
        lfm2_stack(B)
    return B


# LFM2-700M's attention layers (the other 10 of its 16 are short-conv layers).
LFM2_ATTENTION_LAYERS = (2, 5, 8, 10, 12, 14)


def lfm2_stack(B, n_layers: int = 16):
    """the row ops of LFM2-700M's 16 layers (10 short-conv, 6
    attention, in the model's order) over one 1024-token prefill, as the
    driver issues them (lfm2.rs:560-632) with the contractions elided: each
    projection's output is a fixed random buffer (bcx for the conv
    in-projection, o for the out / o / down projections).  Per layer: rms_norm;
    the conv block (h = B*x, conv, ring, C*co) or qk_norm(q), qk_norm(k), rope;
    add; rms_norm; silu_mul; add.  The backend fuses each add with the
    rms_norm after it and the q/k norms with RoPE; the bytes counted are those
    fused ops' compulsory reads and writes."""
    wk = W.LFM2_700M
    b = B.b
    R, H, Q, KV, I, hd, k = wk.rows, wk.dim, wk.q_dim, wk.kv_dim, wk.hidden, wk.head, wk.conv_k
    x, xb, o = B.buf(R * H), B.b.alloc(R * H), B.buf(R * H, 0.01)
    bcx, cy = B.buf(R * 3 * H), b.alloc(R * H)
    q, kk, gate, up = B.buf(R * Q), B.buf(R * KV), B.buf(R * I), B.buf(R * I)
    w_op, w_ffn = b.upload(np.ones(H, np.float32)), b.upload(np.ones(H, np.float32))
    wq, wkk = b.upload(np.ones(hd, np.float32)), b.upload(np.ones(hd, np.float32))
    conv = {l: (B.buf(H * k, 0.3), b.alloc((k - 1) * H)) for l in range(n_layers) if l not in LFM2_ATTENTION_LAYERS}
    pos = np.arange(R, dtype=np.uint64)
    b.rope_prepare(wk.theta, hd, R)
    x0, gate0 = b.alloc(R * H), b.alloc(R * I)
    b.copy(x, 0, x0, 0, R * H)
    b.copy(gate, 0, gate0, 0, R * I)

    def setup():  # the stack's in-place inputs back to their start
        b.copy(x0, 0, x, 0, R * H)
        b.copy(gate0, 0, gate, 0, R * I)

    def stack():
        for l in range(n_layers):
            b.rms_norm(xb, x, w_op, R, H, wk.eps)
            if l in LFM2_ATTENTION_LAYERS:
                b.qk_norm(q, R, Q, hd, wq, wk.eps)
                b.qk_norm(kk, R, KV, hd, wkk, wk.eps)
                b.rope(q, kk, Q, KV, R, pos, hd, wk.theta, False)
            else:
                kern, ring = conv[l]
                b.lfm2_conv_block(bcx, kern, ring, cy, R, H, k)
            b.add_in_place(x, o, R * H)
            b.rms_norm(xb, x, w_ffn, R, H, wk.eps)
            b.silu_mul(gate, up, R * I)
            b.add_in_place(x, o, R * H)

    f = 4
    n_attn = sum(1 for l in range(n_layers) if l in LFM2_ATTENTION_LAYERS)
    nbytes = R * (2 * f * H                      # the first rms_norm: x read, xb written
                  + (2 * n_layers - 1) * 4 * f * H  # each add + rms_norm pair: x, o read; x, xb written
                  + 3 * f * H                    # the last add: x, o read; x written
                  + (n_layers - n_attn) * 4 * f * H  # conv block: bcx read, cy written
                  + n_attn * 2 * f * (Q + KV)    # q/k norms + RoPE: q, k read and written
                  + n_layers * 3 * f * I)        # SwiGLU: gate, up read; gate written
    B.time(f"lfm2 layer stack: {wk.name} ({n_layers} layers: {n_layers - n_attn} conv + {n_attn} attention, "
           f"{R} rows, row ops)", stack, nbytes, setup=setup,
           note="contractions elided (fixed projection outputs)")
    # One of four ranks' share of a conv block when the sequence is split on
    # rows (W.conv_shards): 256 rows and the 2 rows of h before them.
    seg = [sg for sg in W.conv_shards([R], 4, 1, k)][0]
    _, lo, hi, halo, _ = seg
    kern, _ = conv[0]
    shard_cy = b.alloc((hi - lo) * H)
    bcx_shard = b.alloc((hi - lo + halo) * 3 * H)
    b.copy(bcx, (lo - halo) * 3 * H, bcx_shard, 0, (hi - lo + halo) * 3 * H)
    B.time(f"lfm2 layer stack: conv block shard ({hi - lo} rows + {halo}-row halo, rank 1 of 4)",
           lambda: b.lfm2_conv_block_halo(bcx_shard, kern, 0, shard_cy, hi - lo, H, k, halo),
           (hi - lo + halo) * 3 * H * f + (hi - lo) * H * f)


def model_decode(B, n_layers: int = 24, pos: int = 511, samples: int = 50):
    """A whole SmolLM2-1.7B decode step on the device through the trait ops in
    the driver's order (llama.rs decode: per layer rms_norm, project_qkv, RoPE,
    kv_write, attention, o projection, residual add, rms_norm, project_gate_up,
    SwiGLU, down projection, residual add; then the final norm,
    the tied classifier and read()), random bf16 weights, the cache filled to
    `pos`.  Host wall clock per token."""
    import torch

    b = B.b
    wk = W.SMOLLM2_17B_DECODE
    H, Q, KV, I, hd = wk.dim, wk.q_dim, wk.kv_dim, wk.hidden, wk.head
    g = torch.Generator(device="cuda:0").manual_seed(11)

    def mat(o, i):
        t = (torch.randn(o, i, device="cuda:0", generator=g) * (1.0 / i ** 0.5)).to(torch.bfloat16)
        return b.prepare_matrix(BF16, t.view(torch.int16).cpu().numpy().view(np.uint16), None, o, i)

    layers = [dict(q=mat(Q, H), k=mat(KV, H), v=mat(KV, H), o=mat(H, Q), gate=mat(I, H), up=mat(I, H),
                   down=mat(H, I)) for _ in range(n_layers)]
    emb = (torch.randn(wk.vocab, H, device="cuda:0", generator=g) * 0.02).to(torch.bfloat16)
    emb_h = emb.view(torch.int16).cpu().numpy().view(np.uint16)
    b.prepare_embedding(BF16, emb_h, None, wk.vocab, H)
    cls = b.prepare_matrix(BF16, emb_h, None, wk.vocab, H)
    seq = 4096
    b.kv_prepare(n_layers, KV, seq)
    ones = b.upload(np.ones(H, np.float32))
    x, xb, q, k, v, att_o, o = (b.alloc(n) for n in (H, H, Q, KV, KV, Q, H))
    gt, up, dn = b.alloc(I), b.alloc(I), b.alloc(H)
    att = b.alloc(wk.n_heads * seq)
    logits = b.alloc(wk.vocab)
    kf, vf = B.buf(pos * KV), B.buf(pos * KV)
    for layer in range(n_layers):  # the cache up to pos - 1
        b.kv_write(layer, np.arange(pos, dtype=np.uint64), kf, vf, pos)
    out = np.empty(wk.vocab, np.float32)
    kv_mul = wk.n_heads // wk.n_kv_heads

    def step(p):
        b.embed(7, x, 0)
        for L in layers:
            b.rms_norm(xb, x, ones, 1, H, wk.eps)
            b.project_qkv(L["q"], L["k"], L["v"], xb, q, k, v, 1)
            b.rope(q, k, Q, KV, 1, [p], hd, wk.theta, False)
            b.kv_write(layers.index(L), [p], k, v, 1)
            b.attention(q, att_o, att, layers.index(L), [(0, p, 0, 0)], wk.n_heads, kv_mul, hd, KV, seq)
            b.project(L["o"], att_o, o, 1)
            b.add_in_place(x, o, H)
            b.rms_norm(xb, x, ones, 1, H, wk.eps)
            b.project_gate_up(L["gate"], L["up"], xb, gt, up, 1)
            b.silu_mul(gt, up, I)
            b.project(L["down"], gt, dn, 1)
            b.add_in_place(x, dn, H)
        b.rms_norm(xb, x, ones, 1, H, wk.eps)
        b.logits(cls, xb, logits)
        b.read_into(logits, out)

    for exact in (True, False):
        # tolerance mode: every projection and the classifier as warp sums
        b.set_exact(exact)
        try:
            for _ in range(3):
                step(pos)
            times = []
            for _ in range(samples):
                t0 = time.perf_counter()
                step(pos)
                times.append((time.perf_counter() - t0) * 1e3)
        finally:
            b.set_exact(True)
        times.sort()
        mode = "" if exact else ", tolerance mode"
        B.rows.append({"name": f"decode token, SmolLM2-1.7B ({n_layers} layers, bf16, pos {pos}{mode}): trait ops + read()",
                       "ms": None, "us_p10": times[len(times) // 10] * 1e3, "us_median": times[len(times) // 2] * 1e3,
                       "gbs": None, "frac": None, "launches": None,
                       "note": f"host wall clock, {samples} samples; {1e3 / times[len(times) // 2]:.0f} tokens/s"})


def load_table(B, vocab: int = 49152, dim: int = 2048, samples: int = 5):
    """SmolLM2-1.7B's token embedding (bf16) read from a safetensors file into
    bf16 storage (bits handed over) and into Q8_0 (widened and quantised on the
    device).  Host wall clock per call with the file in the page cache."""
    import tempfile

    rng = np.random.default_rng(5)
    bits = (rng.standard_normal((vocab, dim), dtype=np.float32) * np.float32(0.02)).view(np.uint32)
    table = (bits >> np.uint32(16)).astype(np.uint16)
    header = json.dumps({"model.embed_tokens.weight": {"dtype": "BF16", "shape": [vocab, dim],
                                                       "data_offsets": [0, table.nbytes]}}).encode()
    nbytes = table.nbytes
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "model.safetensors")
        with open(path, "wb") as f:
            f.write(len(header).to_bytes(8, "little") + header)
            f.write(table.tobytes())
        del table, bits
        for storage, label in ((BF16, "bf16 (bits handed over)"),
                               (Q8_0, "q8_0 (widened and quantised on the device)")):
            B.b.prepare_embedding_file(path, "model.embed_tokens.weight", storage)
            times = []
            for _ in range(samples):
                t0 = time.perf_counter()
                B.b.prepare_embedding_file(path, "model.embed_tokens.weight", storage)
                times.append(time.perf_counter() - t0)
            times.sort()
            ms = times[len(times) // 2] * 1e3
            B.rows.append({"name": f"prepare_embedding_file {vocab}x{dim} bf16 file -> {label}", "ms": ms,
                           "gbs": nbytes / (ms * 1e-3) / 1e9, "frac": None, "launches": 0,
                           "note": f"host wall clock, {samples} calls, file in the page cache; GB/s of file bytes"})


# FP32 multiply + add pairs per second a B200 issues on its CUDA cores
# (148 SMs x 128 lanes x 1.965 GHz / 2 instructions per pair): the ceiling of
# an exact-order dot, which cannot fuse the multiply into the add.
EXACT_MAC_PEAK = 148 * 128 * 1.965e9 / 2


def contractions(B):
    b = B.b
    rng = np.random.default_rng(5)
    H = 2048
    wq = rng.standard_normal((H, H), dtype=np.float32) * np.float32(0.02)
    wq16 = (wq.view(np.uint32) >> 16).astype(np.uint16)  # bf16 by truncation: any bit pattern will do
    mq = b.prepare_matrix(BF16, wq16, None, H, H)
    for rows in (1, 512):
        x, y = B.buf(rows * H), b.alloc(rows * H)
        macs = rows * H * H
        r = B.time(f"project bf16 {H}x{H}, {rows} row{'s' if rows > 1 else ''}", lambda: b.project(mq, x, y, rows),
                   H * H * 2 + rows * H * 8,
                   note="bound by each output's 2048-long add chain" if rows == 1 else "")
        if r is not None and rows > 1:
            r["note"] = f"{macs / (r['ms'] / 1e3) / 1e12:.2f} T MAC/s = {macs / (r['ms'] / 1e3) / EXACT_MAC_PEAK:.2f} of the exact-order FP32 ceiling"

    def bf16_mat(o, i):
        m = (rng.standard_normal((o, i), dtype=np.float32) * np.float32(0.02)).view(np.uint32) >> 16
        return b.prepare_matrix(BF16, m.astype(np.uint16), None, o, i)

    # tolerance mode (kernrt_cuda_set_exact(ctx, 0)): prefill projections on the
    # tensor cores, x split into bf16 hi + lo inside the call
    for o, i, rows in [(H, H, 512), (8192, H, 512), (8192, H, 4096)]:
        if not B.want(f"project bf16 {o}x{i}, {rows} rows, tensor cores"):
            continue
        wm = mq if (o, i) == (H, H) else bf16_mat(o, i)
        x, y = B.buf(rows * i), b.alloc(rows * o)
        b.set_exact(False)
        try:
            r = B.time(f"project bf16 {o}x{i}, {rows} rows, tensor cores (tolerance mode)",
                       lambda: b.project(wm, x, y, rows), o * i * 2 + rows * i * 4 + rows * o * 4)
        finally:
            b.set_exact(True)
        if r is not None:
            r["note"] = (f"{4 * o * i * rows / (r['ms'] / 1e3) / 1e12:.0f} TFLOP/s of tensor work (W.hi and W.lo), "
                         "the split of x included")
    # the decode projections of one SmolLM2-1.7B layer (fused q/k/v and gate/up)
    wk = W.SMOLLM2_17B_DECODE

    mqkv = [bf16_mat(wk.q_dim, H), bf16_mat(wk.kv_dim, H), bf16_mat(wk.kv_dim, H)]
    mgu = [bf16_mat(wk.hidden, H), bf16_mat(wk.hidden, H)]
    mdown = bf16_mat(H, wk.hidden)
    xd = B.buf(wk.hidden)
    yq, yk, yv, yg, yu, yd = (b.alloc(n) for n in (wk.q_dim, wk.kv_dim, wk.kv_dim, wk.hidden, wk.hidden, H))
    B.time("project_qkv decode (3 x 2048x2048 bf16)", lambda: b.project_qkv(*mqkv, xd, yq, yk, yv, 1),
           3 * H * H * 2, note="one launch; chains of 2048")
    B.time("project_gate_up decode (2 x 8192x2048 bf16)", lambda: b.project_gate_up(*mgu, xd, yg, yu, 1),
           2 * wk.hidden * H * 2, note="one launch; chains of 2048")
    B.time("project down decode (2048x8192 bf16)", lambda: b.project(mdown, xd, yd, 1), H * wk.hidden * 2,
           note="chains of 8192")
    # the same in tolerance mode: each output a warp-wide sum
    if B.want("project_qkv decode, tolerance mode", "project_gate_up decode, tolerance mode",
              "project down decode, tolerance mode"):
        b.set_exact(False)
        try:
            B.time("project_qkv decode, tolerance mode", lambda: b.project_qkv(*mqkv, xd, yq, yk, yv, 1),
                   3 * H * H * 2, note="one launch; warp sums")
            B.time("project_gate_up decode, tolerance mode", lambda: b.project_gate_up(*mgu, xd, yg, yu, 1),
                   2 * wk.hidden * H * 2, note="one launch; warp sums")
            B.time("project down decode, tolerance mode", lambda: b.project(mdown, xd, yd, 1), H * wk.hidden * 2,
                   note="warp sums")
        finally:
            b.set_exact(True)
    codes = rng.integers(-127, 128, size=(3072, 1024), dtype=np.int8)
    sc = rng.uniform(1e-4, 1e-2, size=(3072, 32)).astype(np.float32)
    mg = b.prepare_matrix(Q8_0, codes, sc, 3072, 1024)
    x1, y1 = B.buf(1024), b.alloc(3072)
    B.time("project q8_0 3072x1024, 1 row (Qwen3 gate)", lambda: b.project(mg, x1, y1, 1), 3072 * (1024 + 128) + 1024 * 4)
    vocab = 49152
    emb = (rng.standard_normal((vocab, H), dtype=np.float32) * np.float32(0.02)).view(np.uint32) >> 16
    ml = b.prepare_matrix(BF16, emb.astype(np.uint16), None, vocab, H)
    xl, yl = B.buf(H), b.alloc(vocab)
    B.time(f"logits bf16 {vocab}x{H}", lambda: b.logits(ml, xl, yl), vocab * H * 2 + vocab * 4)
    if B.want(f"logits bf16 {vocab}x{H}, tolerance mode"):
        b.set_exact(False)
        try:
            B.time(f"logits bf16 {vocab}x{H}, tolerance mode", lambda: b.logits(ml, xl, yl), vocab * H * 2 + vocab * 4,
                   note="warp sums")
        finally:
            b.set_exact(True)
    # attention: 32 heads x 64, the cache of one layer, seq 4096
    n_heads, head, seq = 32, 64, 4096
    kv_dim = n_heads * head
    b.kv_prepare(1, kv_dim, seq)
    kx, vx = B.buf(512 * kv_dim), B.buf(512 * kv_dim)
    slots = np.arange(512, dtype=np.uint64)
    B.time("kv_write 512 rows x 2048", lambda: b.kv_write(0, slots, kx, vx, 512), 512 * kv_dim * 16)
    for s0 in range(0, seq, 512):
        b.kv_write(0, slots + s0, kx, vx, 512)
    q1, o1, a1 = B.buf(kv_dim), b.alloc(kv_dim), b.alloc(n_heads * seq)
    B.time("attention decode, 1 row at pos 511 (32x64)", lambda: b.attention(q1, o1, a1, 0, [(0, 511, 0, 0)], n_heads, 1,
                                                                           head, kv_dim, seq),
           512 * kv_dim * 8 + 32 * 512 * 4)
    B.time("attention decode, 1 row at pos 4095 (32x64)",
           lambda: b.attention(q1, o1, a1, 0, [(0, 4095, 0, 0)], n_heads, 1, head, kv_dim, seq),
           4096 * kv_dim * 8 + 32 * 4096 * 4)
    rows = 512
    qp, op, ap = B.buf(rows * kv_dim), b.alloc(rows * kv_dim), b.alloc(rows * n_heads * seq)
    wins = [(0, r, 0, 0) for r in range(rows)]
    B.time("attention prefill, 512 causal rows (32x64)",
           lambda: b.attention(qp, op, ap, 0, wins, n_heads, 1, head, kv_dim, seq), None,
           note="row-tiled scores (16 rows x 64 positions per CTA), then per-(row, head) softmax and sums in order")
    if B.want("attention, tolerance mode"):
        b.set_exact(False)
        try:
            for p in (511, 4095):
                B.time(f"attention decode, 1 row at pos {p} (32x64), tolerance mode",
                       lambda: b.attention(q1, o1, a1, 0, [(0, p, 0, 0)], n_heads, 1, head, kv_dim, seq),
                       (p + 1) * kv_dim * 8 + 32 * (p + 1) * 4, note="chunks of 64 positions, then combined")
        finally:
            b.set_exact(True)


def chain_time(B, wk):
    import torch

    b = B.b
    R = wk.rows
    if wk.storage == "bf16":
        t = (torch.randn(wk.vocab, wk.dim, device="cuda:0", generator=B.g) * 0.02).to(torch.bfloat16)
        b.prepare_embedding(BF16, t.view(torch.int16).cpu().numpy().view(np.uint16), None, wk.vocab, wk.dim)
    elif wk.storage == "q8_0":
        rng = np.random.default_rng(2)
        codes = rng.integers(-127, 128, size=(wk.vocab, wk.dim), dtype=np.int8)
        sc = rng.uniform(1e-4, 1e-2, size=(wk.vocab, wk.dim // 32)).astype(np.float32)
        b.prepare_embedding(Q8_0, codes, sc, wk.vocab, wk.dim)
    h = {n: B.buf(R * n_) for n, n_ in [("q", wk.q_dim), ("k", wk.kv_dim), ("gate", wk.hidden), ("up", wk.hidden),
                                         ("resid", wk.dim)]}
    h["gate0"] = b.alloc(R * wk.hidden)
    b.copy(h["gate"], 0, h["gate0"], 0, R * wk.hidden)
    h["x"] = B.buf(R * wk.dim) if wk.storage == "none" else b.alloc(R * wk.dim)
    h["xb"] = b.alloc(R * wk.dim)
    h["w_att"] = b.upload(np.ones(wk.dim, np.float32))
    kw = {}
    if wk.storage != "none":
        kw["tokens"] = b.upload_bytes(np.random.default_rng(3).integers(0, wk.vocab, R).astype(np.int32))
    kw["positions"] = b.upload_bytes(wk.positions())
    if wk.qk_norm:
        kw["w_q"] = b.upload(np.ones(wk.head, np.float32))
        kw["w_k"] = b.upload(np.ones(wk.head, np.float32))
    nb = (wk.dim + 31) // 32
    if wk.final_q8:
        kw.update(w_final=b.upload(np.ones(wk.dim, np.float32)), codes=b.alloc_bytes(R * nb * 32),
                  scales=b.alloc_bytes(R * nb * 4), scales_f16=b.alloc_bytes(R * nb * 2))
    b.rope_prepare(wk.theta, wk.head, wk.seq_len + wk.pos0)
    args = dict(rows=R, dim=wk.dim, q_dim=wk.q_dim, kv_dim=wk.kv_dim, hidden=wk.hidden, head_size=wk.head,
                eps=wk.eps, theta=wk.theta, final_eps=wk.eps, x=h["x"], xb=h["xb"], w_att=h["w_att"],
                q=h["q"], k=h["k"], gate=h["gate"], up=h["up"], resid=h["resid"], **kw)
    x0 = None
    if wk.storage == "none":
        x0 = b.alloc(R * wk.dim)
        b.copy(h["x"], 0, x0, 0, R * wk.dim)

    def setup():
        b.copy(h["gate0"], 0, h["gate"], 0, R * wk.hidden)
        if x0 is not None:
            b.copy(x0, 0, h["x"], 0, R * wk.dim)

    B.time(f"chain: {wk.name} ({R} rows)", lambda: b.layer_chain(**args), R * wk.bytes_per_row(), setup=setup,
           note="working set below L2" if R * wk.bytes_per_row() < 126e6 else "")


def decode_latency(B):
    """configs[1] decode: one token at position 511 through the row ops of a
    SmolLM2-1.7B block as the driver calls them, with a read() per step."""
    import torch

    b = B.b
    wk = W.SMOLLM2_17B_DECODE
    t = (torch.randn(wk.vocab, wk.dim, device="cuda:0", generator=B.g) * 0.02).to(torch.bfloat16)
    b.prepare_embedding(BF16, t.view(torch.int16).cpu().numpy().view(np.uint16), None, wk.vocab, wk.dim)
    x, xb = b.alloc(wk.dim), b.alloc(wk.dim)
    q, k, o = B.buf(wk.q_dim), B.buf(wk.kv_dim), B.buf(wk.dim)
    g, u = B.buf(wk.hidden), B.buf(wk.hidden)
    w = b.upload(np.ones(wk.dim, np.float32))
    out = np.empty(wk.dim, np.float32)
    samples = []
    for i in range(300 + 20):
        t0 = time.perf_counter()
        b.embed(7, x, 0)
        b.rms_norm(xb, x, w, 1, wk.dim, wk.eps)
        b.rope(q, k, wk.q_dim, wk.kv_dim, 1, [511], wk.head, wk.theta, False)
        b.add_in_place(x, o, wk.dim)
        b.rms_norm(xb, x, w, 1, wk.dim, wk.eps)
        b.silu_mul(g, u, wk.hidden)
        b.add_in_place(x, o, wk.dim)
        b.read_into(x, out)
        if i >= 20:
            samples.append((time.perf_counter() - t0) * 1e6)
    samples.sort()
    B.rows.append({"name": "decode step, 1 row (configs[1], pos 511): row ops + read()", "ms": None,
                   "us_p10": samples[len(samples) // 10], "us_median": samples[len(samples) // 2], "gbs": None,
                   "frac": None, "launches": None, "note": "host wall clock, 300 samples"})


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--reps", type=int, default=10)
    p.add_argument("--json", action="store_true")
    p.add_argument("--only", default=None, help="regex: time only the ops whose name matches")
    args = p.parse_args()
    B = run(args.reps, args.only)
    if args.json:
        for r in B.rows:
            print(json.dumps(r))
        return
    print(f"| op | ms (median) | GB/s | of {B.peak:.0f} GB/s | launches | note |")
    print("|---|---:|---:|---:|---:|---|")
    for r in B.rows:
        if r.get("ms") is None:
            print(f"| {r['name']} | p10 {r['us_p10']:.1f} us, median {r['us_median']:.1f} us | | | | {r['note']} |")
            continue
        gbs = "" if r["gbs"] is None else f"{r['gbs']:.0f}"
        frac = "" if r["frac"] is None else f"{r['frac']:.3f}"
        print(f"| {r['name']} | {r['ms']:.4f} | {gbs} | {frac} | {r['launches']:.0f} | {r['note']} |")


if __name__ == "__main__":
    main()
