"""The layer-op workloads the backend is measured and checked on.

Shapes follow the model families KernRT drives (SmolLM2 / Llama, Qwen3, LFM2;
src/arch/llm/llama.rs:26-67, lfm2.rs) at the sizes of the benchmark
configurations: every entry is one Llama-family block's row-op chain
(embed -> RMSNorm -> [q/k norm] -> RoPE(Q, K) -> SwiGLU -> residual add
[-> final RMSNorm + Q8_0]) or the LFM2 short-conv block.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Workload:
    name: str
    vocab: int
    dim: int
    n_heads: int
    n_kv_heads: int
    head: int
    hidden: int
    theta: float
    eps: float
    storage: str          # embedding storage: "bf16" | "q8_0" | "none" (x is an input)
    rows: int
    seq_len: int          # positions are row % seq_len (+ pos0)
    pos0: int = 0
    qk_norm: bool = False
    final_q8: bool = False
    conv_k: int = 0       # LFM2 short-conv taps (0 = no conv block)

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head

    def positions(self, lo: int = 0, hi: int | None = None) -> np.ndarray:
        hi = self.rows if hi is None else hi
        r = np.arange(lo, hi, dtype=np.int64)
        return (self.pos0 + r % self.seq_len).astype(np.int32)

    def bytes_per_row(self) -> int:
        """Compulsory HBM bytes of the fused chain per token row: each
        activation row read and/or written once, the embedding row read once
        in its stored width; norm weights and the RoPE table (L2-resident) are
        not counted."""
        f = 4
        b = 0
        if self.storage == "bf16":
            b += 2 * self.dim
        elif self.storage == "q8_0":
            b += self.dim + 4 * (self.dim // 32)
        else:
            b += f * self.dim                     # x read
        b += f * self.dim                         # xb written
        b += 2 * f * self.q_dim + 2 * f * self.kv_dim  # Q, K read + written
        b += 3 * f * self.hidden                  # gate, up read; gate written
        b += 2 * f * self.dim                     # residual read; x written
        if self.final_q8:
            nb = (self.dim + 31) // 32
            b += 32 * nb + 4 * nb                 # codes + f32 scales
        return b

    def stage_bytes_per_row(self, two_pass: bool = False) -> dict:
        """The same compulsory bytes split by the stage that moves them when
        the chain runs as the norm stage plus the RoPE/SwiGLU stream.  With
        the two-pass norm stage (gathered bf16 / f32 rows) the norm stage
        only reads the gathered row for the row scales and the stream kernel
        moves everything else (its second read of the gathered row is traffic
        beyond the compulsory bytes, so it is not counted)."""
        f = 4
        stream = 2 * f * self.q_dim + 2 * f * self.kv_dim + 3 * f * self.hidden
        if two_pass:
            gathered = (2 if self.storage == "bf16" else f) * self.dim
            return {"norm": gathered, "stream": self.bytes_per_row() - gathered}
        return {"norm": self.bytes_per_row() - stream, "stream": stream}


SMOLLM2_135M = Workload("smollm2-135m-prefill128", 49152, 576, 9, 3, 64, 1536, 1e5, 1e-5, "bf16",
                        rows=128, seq_len=128)
SMOLLM2_17B_DECODE = Workload("smollm2-1.7b-decode", 49152, 2048, 32, 32, 64, 8192, 1.3e5, 1e-5,
                              "bf16", rows=1, seq_len=1, pos0=511)
SMOLLM2_17B_PREFILL = Workload("smollm2-1.7b-prefill512", 49152, 2048, 32, 32, 64, 8192, 1.3e5, 1e-5,
                               "bf16", rows=512, seq_len=512)
QWEN3_06B_Q8 = Workload("qwen3-0.6b-q8_0-prefill256", 151936, 1024, 16, 8, 128, 3072, 1e6, 1e-6, "q8_0",
                        rows=256, seq_len=256, qk_norm=True, final_q8=True)
LFM2_700M = Workload("lfm2-700m-prefill1024", 65536, 1536, 24, 8, 64, 4608, 1e6, 1e-5, "none",
                     rows=1024, seq_len=1024, qk_norm=True, conv_k=3)
# The headline: 16 sequences x 4096 rows through the SmolLM2-1.7B chain.
SMOLLM2_17B_65K = Workload("smollm2-1.7b-chain-65536rows", 49152, 2048, 32, 32, 64, 8192, 1.3e5, 1e-5,
                           "bf16", rows=65536, seq_len=4096)

ALL = [SMOLLM2_135M, SMOLLM2_17B_DECODE, SMOLLM2_17B_PREFILL, QWEN3_06B_Q8, LFM2_700M, SMOLLM2_17B_65K]


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, as-even-as-possible row range [lo, hi) of `rank` among
    `world` ranks (token rows are independent, so no exchange is needed)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def conv_shards(seq_lens, world: int, rank: int, k: int) -> list[tuple[int, int, int, int, bool]]:
    """The LFM2 short-conv rows of `rank` when the concatenated sequences
    (lengths `seq_lens`) are split into contiguous row blocks (shard_rows): a
    list of (sequence, lo, hi, halo, ends) segments, rows [lo, hi) of that
    sequence.  The causal conv of row r reads h of rows r - k + 1 .. r of its
    own sequence (lfm2.rs:584-624), so a segment that starts inside a sequence
    takes halo = min(k - 1, lo) preceding rows of it, staged locally with the
    segment before the run; `ends` marks the segment holding the sequence's
    last row, the one that seeds the decode ring (lfm2.rs:601-610)."""
    total = sum(seq_lens)
    lo_r, hi_r = shard_rows(total, world, rank)
    out, start = [], 0
    for i, n in enumerate(seq_lens):
        lo, hi = max(lo_r, start) - start, min(hi_r, start + n) - start
        if lo < hi:
            out.append((i, lo, hi, min(k - 1, lo), hi == n))
        start += n
    return out

