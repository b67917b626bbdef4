"""Seeded synthetic inputs for the parity tests.

The uniform generator is KernRT's own test LCG (tests/backends.rs:41-51,
src/ops/mod.rs:49-60): ``s = s*6364136223846793005 + 1442695040888963407``,
``u = (s >> 40) / 2^24 - 0.5``.  Normals are Box-Muller over two LCG streams.
Vectorised with jump-ahead, so large fills stay fast and bit-identical to the
sequential definition.
"""
from __future__ import annotations

import numpy as np

_A = np.uint64(6364136223846793005)
_C = np.uint64(1442695040888963407)


def lcg_states(seed: int, count: int) -> np.ndarray:
    """States s_1..s_count of the LCG started at `seed` (uint64, wrapping)."""
    out = np.empty(count, np.uint64)
    if count == 0:
        return out
    with np.errstate(over="ignore"):
        out[0] = np.uint64(seed) * _A + _C
        filled = 1
        a_m, c_m = _A, _C  # one step: s -> a*s + c
        while filled < count:
            n = min(filled, count - filled)
            out[filled:filled + n] = out[:n] * a_m + c_m
            filled += n
            # compose the m-step map with itself: m -> 2m
            c_m = c_m * a_m + c_m
            a_m = a_m * a_m
    return out


def lcg_uniform(count: int, seed: int) -> np.ndarray:
    """KernRT's `fill`/`random`: f32 in [-0.5, 0.5)."""
    s = lcg_states(seed, count)
    return ((s >> np.uint64(40)).astype(np.float32) / np.float32(1 << 24)) - np.float32(0.5)


def lcg_normal(count: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    u1 = lcg_uniform(count, seed).astype(np.float64) + 0.5
    u2 = lcg_uniform(count, seed + 0x9E3779B9).astype(np.float64) + 0.5
    z = np.sqrt(-2.0 * np.log1p(-u1)) * np.cos(2.0 * np.pi * u2)
    return (mean + std * z).astype(np.float32)


def tokens(count: int, vocab: int, seed: int) -> np.ndarray:
    s = lcg_states(seed, count)
    return ((s >> np.uint64(33)) % np.uint64(vocab)).astype(np.int32)


def bf16_table(vocab: int, dim: int, seed: int, std: float = 0.02) -> np.ndarray:
    from oracle.oracle import f32_to_bf16_bits

    return f32_to_bf16_bits(lcg_normal(vocab * dim, seed, 0.0, std)).reshape(vocab, dim)


def q8_table(vocab: int, dim: int, seed: int):
    """Q8_0 codes uniform in [-127, 127] and block scales ~U(1e-4, 1e-2)."""
    s = lcg_states(seed, vocab * dim)
    codes = (((s >> np.uint64(33)) % np.uint64(255)).astype(np.int64) - 127).astype(np.int8)
    u = lcg_uniform(vocab * dim // 32, seed + 7).astype(np.float64) + 0.5
    scales = (1e-4 + u * (1e-2 - 1e-4)).astype(np.float32)
    return codes.reshape(vocab, dim), scales.reshape(vocab, dim // 32)


def bf16_table_fast(vocab: int, dim: int, seed: int, std: float = 0.02) -> np.ndarray:
    """Large bf16 tables (full vocabularies): numpy's PCG64 normals, RNE to bf16."""
    from oracle.oracle import f32_to_bf16_bits

    rng = np.random.default_rng(seed)
    out = np.empty((vocab, dim), np.uint16)
    step = max(1, (1 << 24) // dim)
    for lo in range(0, vocab, step):
        hi = min(vocab, lo + step)
        v = rng.standard_normal((hi - lo, dim), dtype=np.float32) * np.float32(std)
        out[lo:hi] = f32_to_bf16_bits(v)
    return out


def q8_table_fast(vocab: int, dim: int, seed: int):
    rng = np.random.default_rng(seed)
    codes = rng.integers(-127, 128, size=(vocab, dim), dtype=np.int8)
    scales = rng.uniform(1e-4, 1e-2, size=(vocab, dim // 32)).astype(np.float32)
    return codes, scales


def safetensors_bytes(tensors, metadata=None) -> bytes:
    """A safetensors image (src/formats/safetensors.rs:1-16): u64 LE header
    length, the JSON header, then the payloads in the given order.  `tensors`
    is a list of (name, dtype, shape, payload_bytes)."""
    import json

    header, data = {}, b""
    for name, dtype, shape, payload in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [len(data), len(data) + len(payload)]}
        data += payload
    if metadata is not None:
        header["__metadata__"] = metadata
    hb = json.dumps(header).encode()
    return len(hb).to_bytes(8, "little") + hb + data


def safetensors_raw(header_text: bytes, data: bytes = b"") -> bytes:
    """A safetensors image around an exact header text (for malformed headers)."""
    return len(header_text).to_bytes(8, "little") + header_text + data
