"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle is a plain-C restatement of KernRT's scalar `reference` backend
(``oracle/kernrt_oracle.c``; each C function cites the Rust file:line it
follows).  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline / reference arm use this module, always as the checker or as the
timed CPU baseline, never as part of the CUDA product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libkernrt_oracle.so")

F32, BF16, Q8_0, Q8_0X4 = 0, 1, 2, 3
Q8_BLOCK = 32

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc only) and return the .so path."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "kernrt_oracle.c")
        if not os.path.exists(LIB_PATH) or (
            os.path.exists(src) and os.path.getmtime(src) > os.path.getmtime(LIB_PATH)
        ):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
SZ = C.c_size_t


class Chain(C.Structure):
    """Mirror of ``kro_chain`` in kernrt_oracle.c."""

    _fields_ = [
        ("rows", SZ), ("dim", SZ), ("q_dim", SZ), ("kv_dim", SZ), ("hidden", SZ), ("head", SZ),
        ("eps", C.c_float), ("theta", C.c_float), ("final_eps", C.c_float),
        ("interleaved", C.c_int),
        ("t_kind", C.c_int), ("t_vocab", SZ), ("t_dim", SZ), ("t_data", P), ("t_scales", P),
        ("tokens", P), ("positions", P), ("w_att", P), ("w_q", P), ("w_k", P), ("w_final", P),
        ("x", P), ("xb", P), ("q", P), ("k", P), ("gate", P), ("up", P), ("resid", P),
        ("codes", P), ("scales", P), ("scales_f16", P),
    ]


def _declare(L: C.CDLL) -> None:
    L.kro_bf16_to_f32.restype = C.c_float
    L.kro_bf16_to_f32.argtypes = [C.c_uint16]
    L.kro_f32_to_bf16_bits.restype = C.c_uint16
    L.kro_f32_to_bf16_bits.argtypes = [C.c_float]
    L.kro_f32_to_f16_bits.restype = C.c_uint16
    L.kro_f32_to_f16_bits.argtypes = [C.c_float]
    L.kro_f16_scale_to_f32.restype = C.c_float
    L.kro_f16_scale_to_f32.argtypes = [C.c_uint16]
    L.kro_q8_quantize_into.argtypes = [P, SZ, P, P, P]
    L.kro_q8_0x4_pack.restype = C.c_int
    L.kro_q8_0x4_pack.argtypes = [P, SZ, SZ, P]
    L.kro_q8_0x4_to_row_major.argtypes = [P, SZ, SZ, P, P]
    L.kro_embed_rows.argtypes = [C.c_int, P, P, SZ, SZ, P, SZ, P]
    L.kro_rms_norm.argtypes = [P, P, P, SZ, SZ, C.c_float]
    L.kro_qk_norm.argtypes = [P, SZ, SZ, SZ, P, C.c_float]
    L.kro_rope.argtypes = [P, P, SZ, SZ, SZ, P, SZ, C.c_float, C.c_int]
    L.kro_silu_mul.argtypes = [P, P, SZ]
    L.kro_add_in_place.argtypes = [P, P, SZ]
    L.kro_mul.argtypes = [P, SZ, P, SZ, P, SZ, SZ]
    L.kro_copy.argtypes = [P, SZ, P, SZ, SZ]
    L.kro_conv_prefill.argtypes = [P, P, P, SZ, SZ, SZ]
    L.kro_conv_decode.argtypes = [P, P, P, P, SZ, SZ]
    L.kro_lfm2_conv_block.argtypes = [P, P, P, P, P, P, SZ, SZ, SZ]
    L.kro_project.argtypes = [C.c_int, P, P, SZ, SZ, P, SZ, P, C.c_int]
    L.kro_kv_write.argtypes = [P, P, SZ, SZ, SZ, P, SZ, P, P, SZ]
    L.kro_attention.argtypes = [P, P, P, P, P, SZ, P, SZ, SZ, SZ, SZ, SZ, SZ]
    L.kro_chain_run.argtypes = [C.POINTER(Chain)]
    L.kro_chain_run_mt.argtypes = [C.POINTER(Chain), C.c_int]
    L.kro_chain_struct_size.restype = SZ
    L.kro_max_threads.restype = C.c_int
    assert L.kro_chain_struct_size() == C.sizeof(Chain), "kro_chain layout drifted"


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# --- number formats -----------------------------------------------------------

def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(v: np.ndarray) -> np.ndarray:
    """Vectorised restatement of the C function (src/ops/quant.rs:707-711)."""
    b = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32)
    lsb = (b >> np.uint32(16)) & np.uint32(1)
    with np.errstate(over="ignore"):
        return ((b + np.uint32(0x7FFF) + lsb) >> np.uint32(16)).astype(np.uint16)  # u32 wrapping add


def f32_to_f16_bits(v: float) -> int:
    return lib().kro_f32_to_f16_bits(float(v))


def f16_scale_to_f32(bits: int) -> float:
    return lib().kro_f16_scale_to_f32(int(bits))


# --- Q8_0 ----------------------------------------------------------------------

def q8_quantize(x: np.ndarray):
    """Q8Vec::quantize_into of one vector -> (quants, scales, scales_f16)."""
    x = f32(x).ravel()
    blocks = (x.size + Q8_BLOCK - 1) // Q8_BLOCK
    q = np.zeros(blocks * Q8_BLOCK, np.int8)
    s = np.zeros(blocks, np.float32)
    h = np.zeros(blocks, np.uint16)
    lib().kro_q8_quantize_into(_p(x), x.size, _p(q), _p(s), _p(h))
    return q, s, h


def q8_quantize_rows(x: np.ndarray):
    """Row-wise quantize of a [rows, dim] matrix -> codes [rows, blocks*32], scales, f16."""
    x = f32(x)
    rows, dim = x.shape
    blocks = (dim + Q8_BLOCK - 1) // Q8_BLOCK
    q = np.zeros((rows, blocks * Q8_BLOCK), np.int8)
    s = np.zeros((rows, blocks), np.float32)
    h = np.zeros((rows, blocks), np.uint16)
    L = lib()
    for r in range(rows):
        L.kro_q8_quantize_into(_p(x[r]), dim, _p(q[r]), _p(s[r]), _p(h[r]))
    return q, s, h


def q8_0_from_f32(w: np.ndarray):
    """Matrix::from_f32_q8_0 (src/ops/quant.rs:544-557): quantize the flattened
    tensor in 32-blocks -> (quants [out*in], scales [out*in/32])."""
    w = f32(w)
    assert w.shape[1] % Q8_BLOCK == 0
    q, s, _ = q8_quantize(w.ravel())
    return q.reshape(w.shape), s.reshape(w.shape[0], -1)


def q8_0x4_pack(w: np.ndarray) -> np.ndarray:
    w = f32(w)
    out_dim, in_dim = w.shape
    blocks = np.zeros((out_dim // 4) * (in_dim // Q8_BLOCK) * 136, np.uint8)
    rc = lib().kro_q8_0x4_pack(_p(w), out_dim, in_dim, _p(blocks))
    assert rc == 0
    return blocks


def q8_0x4_to_row_major(blocks: np.ndarray, out_dim: int, in_dim: int):
    q = np.zeros((out_dim, in_dim), np.int8)
    s = np.zeros((out_dim, in_dim // Q8_BLOCK), np.float32)
    lib().kro_q8_0x4_to_row_major(_p(blocks), out_dim, in_dim, _p(q), _p(s))
    return q, s


# --- safetensors payloads and the HF loaders' storage rules ------------------------

def st_f16_to_f32(bits) -> np.ndarray:
    """src/formats/safetensors.rs:365-385 f16_to_f32_local, element by element:
    zero keeps its sign; a subnormal mantissa is shifted left until the
    implicit bit appears, the exponent counting down from 127 - 15 + 1; Inf and
    NaN keep their mantissa bits; normals rebias the exponent."""
    b = np.asarray(bits, dtype=np.uint16).ravel()
    out = np.zeros(b.size, np.uint32)
    for i, v in enumerate(b.tolist()):
        sign = (v >> 15) << 31
        exponent = (v >> 10) & 0x1F
        mantissa = v & 0x3FF
        if exponent == 0 and mantissa == 0:
            w = sign
        elif exponent == 0:
            e = 127 - 15 + 1
            while mantissa & 0x400 == 0:
                mantissa <<= 1
                e -= 1
            w = sign | (e << 23) | ((mantissa & 0x3FF) << 13)
        elif exponent == 0x1F:
            w = sign | 0x7F800000 | (mantissa << 13)
        else:
            w = sign | ((exponent + (127 - 15)) << 23) | (mantissa << 13)
        out[i] = w
    return out.view(np.float32).reshape(np.shape(bits))


def st_widen(dtype: str, raw: np.ndarray) -> np.ndarray:
    """hf.rs:97-107 widen over safetensors.rs:280-300 decode: F32 as is, BF16
    as the top half of an f32, F16 through f16_to_f32_local."""
    if dtype == "F32":
        return f32(raw)
    if dtype == "BF16":
        return bf16_to_f32(raw)
    return st_f16_to_f32(raw)


def table_from_raw(dtype: str, raw: np.ndarray, storage: int):
    """hf.rs:151-191 matrix_from_raw for a [vocab, dim] payload, returned as what
    embed_rows reads: (kind, data, scales).  A bf16 payload is handed over as
    it is for bf16 storage; bf16 is quantised for block-aligned Q8_0 / Q8_0x4;
    otherwise the payload is widened and kept f32, quantised for aligned
    Q8_0x4, or narrowed to bf16 by dropping the low half.  Q8_0x4 reads back
    de-interleaved with its f16 scales widened (quant.rs:198-220)."""
    vocab, dim = raw.shape
    aligned_q8 = dim % Q8_BLOCK == 0
    aligned_q8x4 = aligned_q8 and vocab % 4 == 0

    def q8x4(w):
        q, s = q8_0x4_to_row_major(q8_0x4_pack(w), vocab, dim)
        return Q8_0, q, s

    if dtype == "BF16" and storage == BF16:
        return BF16, np.ascontiguousarray(raw, dtype=np.uint16), None
    if dtype == "BF16" and storage == Q8_0 and aligned_q8:
        q, s = q8_0_from_f32(st_widen(dtype, raw))
        return Q8_0, q, s
    if dtype == "BF16" and storage == Q8_0X4 and aligned_q8x4:
        return q8x4(st_widen(dtype, raw))
    w = st_widen(dtype, raw)
    if storage == F32:
        return F32, w, None
    if storage == Q8_0X4 and aligned_q8x4:
        return q8x4(w)
    return BF16, (np.ascontiguousarray(w).view(np.uint32) >> np.uint32(16)).astype(np.uint16), None


# --- row ops ---------------------------------------------------------------------

def embed_rows(kind: int, data: np.ndarray, scales, vocab: int, dim: int, tokens) -> np.ndarray:
    tokens = np.ascontiguousarray(tokens, dtype=np.int32)
    out = np.zeros((tokens.size, dim), np.float32)
    lib().kro_embed_rows(kind, _p(data), _p(scales), vocab, dim, _p(tokens), tokens.size, _p(out))
    return out


def rms_norm(x, w, eps) -> np.ndarray:
    x = f32(x)
    rows, dim = x.shape
    out = np.empty_like(x)
    lib().kro_rms_norm(_p(out), _p(x), _p(f32(w)), rows, dim, float(eps))
    return out


def qk_norm(v, head, w, eps) -> np.ndarray:
    v = f32(v).copy()
    rows, width = v.shape
    lib().kro_qk_norm(_p(v), rows, width, head, _p(f32(w)), float(eps))
    return v


def rope(q, k, positions, head, theta, interleaved=False):
    q = f32(q).copy()
    k = f32(k).copy()
    pos = np.ascontiguousarray(positions, dtype=np.uint64)
    rows = pos.size
    lib().kro_rope(_p(q), _p(k), q.shape[1], k.shape[1], rows, _p(pos), head, float(theta),
                   int(bool(interleaved)))
    return q, k


def silu_mul(gate, up) -> np.ndarray:
    g = f32(gate).copy()
    u = f32(up)
    lib().kro_silu_mul(_p(g), _p(u), g.size)
    return g


def add_in_place(dst, src) -> np.ndarray:
    d = f32(dst).copy()
    lib().kro_add_in_place(_p(d), _p(f32(src)), d.size)
    return d


def mul_into(out: np.ndarray, out_off, a: np.ndarray, a_off, b: np.ndarray, b_off, length):
    """In-place on `out` (which may be the same array object as a and/or b)."""
    lib().kro_mul(_p(out), out_off, _p(a), a_off, _p(b), b_off, length)


def copy_into(src: np.ndarray, src_off, dst: np.ndarray, dst_off, length):
    lib().kro_copy(_p(src), src_off, _p(dst), dst_off, length)


def conv_prefill(x, kernel, k) -> np.ndarray:
    x = f32(x)
    rows, dim = x.shape
    out = np.zeros_like(x)
    lib().kro_conv_prefill(_p(out), _p(x), _p(f32(kernel)), rows, dim, k)
    return out


def conv_decode(x, kernel, state, k):
    """Returns (out, new_state); does not modify the inputs."""
    x = f32(x).ravel()
    st = f32(state).copy()
    out = np.zeros_like(x)
    lib().kro_conv_decode(_p(out), _p(x), _p(f32(kernel)), _p(st), x.size, k)
    return out, st


def lfm2_conv_block(bcx, kernel, ring, k):
    """Returns (cy, new_ring)."""
    bcx = f32(bcx)
    rows, three_dim = bcx.shape
    dim = three_dim // 3
    ring = f32(ring).copy()
    cy = np.zeros((rows, dim), np.float32)
    h = np.zeros((rows, dim), np.float32)
    co = np.zeros((rows, dim), np.float32)
    lib().kro_lfm2_conv_block(_p(bcx), _p(f32(kernel)), _p(ring), _p(cy), _p(h), _p(co), rows,
                              dim, k)
    return cy, ring


def lfm2_conv_block_shard(bcx, kernel, k, lo, hi, halo):
    """Rows [lo, hi) of one sequence's conv block computed from its rows
    lo - halo .. hi alone (the shard's own rows and its staged halo): the
    oracle's block over those rows, outputs of the halo rows dropped.  With
    halo = min(k - 1, lo) this equals the unsharded block's rows [lo, hi)
    (a row's conv reads only the k - 1 rows before it).  Returns (cy, ring) with
    ring the last k - 1 rows of h over those rows (the sequence's ring when
    hi is its end)."""
    cy, ring = lfm2_conv_block(f32(bcx)[lo - halo:hi], kernel, np.zeros((max(k - 1, 0), f32(bcx).shape[1] // 3),
                                                                        np.float32), k)
    return cy[halo:], ring


def chain(*, dim, q_dim, kv_dim, hidden, head, eps, theta, positions, w_att, q, k, gate, up,
          resid, tokens=None, table=None, x=None, interleaved=False, w_q=None, w_k=None,
          w_final=None, final_eps=None, threads=1, in_place=False):
    """Run the row-op chain of kernrt_oracle.c (kro_chain_run[_mt]).

    `table` is (kind, data, scales, vocab).  Returns a dict of outputs.  With
    in_place=True, q/k/gate (f32, contiguous) are updated in place instead of
    copied first (the timed CPU baseline uses this).
    """
    positions = np.ascontiguousarray(positions, dtype=np.uint64)
    rows = positions.size
    if in_place:
        for a in (q, k, gate):
            assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    else:
        q = f32(q).copy()
        k = f32(k).copy()
        gate = f32(gate).copy()
    up = f32(up)
    resid = f32(resid)
    if tokens is not None:
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        xo = np.zeros((rows, dim), np.float32)
    else:
        xo = f32(x).copy()
    xb = np.zeros((rows, dim), np.float32)
    blocks = (dim + Q8_BLOCK - 1) // Q8_BLOCK
    codes = scales = scales16 = None
    if w_final is not None:
        codes = np.zeros((rows, blocks * Q8_BLOCK), np.int8)
        scales = np.zeros((rows, blocks), np.float32)
        scales16 = np.zeros((rows, blocks), np.uint16)
    keep = []

    def ptr(a):
        if a is None:
            return None
        a = np.ascontiguousarray(a)
        keep.append(a)
        return a.ctypes.data

    c = Chain()
    c.rows, c.dim, c.q_dim, c.kv_dim, c.hidden, c.head = rows, dim, q_dim, kv_dim, hidden, head
    c.eps, c.theta = float(eps), float(theta)
    c.final_eps = float(final_eps if final_eps is not None else eps)
    c.interleaved = int(bool(interleaved))
    if table is not None:
        kind, data, tscales, vocab = table
        c.t_kind, c.t_vocab, c.t_dim = kind, vocab, dim
        c.t_data, c.t_scales = ptr(data), ptr(tscales)
    c.tokens = ptr(tokens)
    c.positions = ptr(positions)
    c.w_att = ptr(f32(w_att))
    c.w_q = ptr(None if w_q is None else f32(w_q))
    c.w_k = ptr(None if w_k is None else f32(w_k))
    c.w_final = ptr(None if w_final is None else f32(w_final))
    c.x, c.xb, c.q, c.k = ptr(xo), ptr(xb), ptr(q), ptr(k)
    c.gate, c.up, c.resid = ptr(gate), ptr(up), ptr(resid)
    c.codes, c.scales, c.scales_f16 = ptr(codes), ptr(scales), ptr(scales16)
    if threads > 1:
        lib().kro_chain_run_mt(C.byref(c), int(threads))
    else:
        lib().kro_chain_run(C.byref(c))
    return {"x": xo, "xb": xb, "q": q, "k": k, "gate": gate, "codes": codes, "scales": scales,
            "scales_f16": scales16}


def max_threads() -> int:
    return lib().kro_max_threads()


# --- contractions (reference.rs:73-79, 151-159, 259-306, 402-482) -----------------------

def project(kind: int, data: np.ndarray, scales, out_dim: int, in_dim: int, x, threads: int = 0) -> np.ndarray:
    """y[r, o] = dot(decode_row(W, o), x[r]) in the reference's order; x is
    [rows, in_dim] f32.  `threads` 0 = every host thread."""
    x = np.ascontiguousarray(f32(x)).reshape(-1, in_dim)
    y = np.zeros((x.shape[0], out_dim), np.float32)
    data = np.ascontiguousarray(data)
    sc = None if scales is None else np.ascontiguousarray(f32(scales))
    lib().kro_project(kind, _p(data), _p(sc), out_dim, in_dim, _p(x), x.shape[0], _p(y),
                      threads or max_threads())
    return y


def kv_write(key_cache: np.ndarray, value_cache: np.ndarray, kv_dim: int, seq_len: int, layer: int,
             slots, k, v, rows: int):
    """Writes rows of k and v into the caches (updated in place and returned)."""
    slots = np.ascontiguousarray(slots, dtype=np.uint64)
    k, v = np.ascontiguousarray(f32(k)), np.ascontiguousarray(f32(v))
    lib().kro_kv_write(_p(key_cache), _p(value_cache), kv_dim, seq_len, layer, _p(slots), slots.size,
                       _p(k), _p(v), rows)
    return key_cache, value_cache


def attention(q, key_cache, value_cache, layer: int, windows, n_heads: int, kv_mul: int, head_size: int,
              kv_dim: int, seq_len: int, att=None):
    """(out, att): windows is a sequence of (att_start, slot, shared_start,
    shared_end); att (rows x n_heads x seq_len) keeps what the call does not
    write."""
    w = np.ascontiguousarray(windows, dtype=np.uint64).reshape(-1, 4)
    rows = w.shape[0]
    q = np.ascontiguousarray(f32(q)).reshape(rows, n_heads * head_size)
    out = np.zeros((rows, n_heads * head_size), np.float32)
    att = np.zeros((rows, n_heads, seq_len), np.float32) if att is None else np.array(att, np.float32)
    lib().kro_attention(_p(q), _p(out), _p(att), _p(np.ascontiguousarray(key_cache)),
                        _p(np.ascontiguousarray(value_cache)), layer, _p(w), rows, n_heads, kv_mul, head_size,
                        kv_dim, seq_len)
    return out, att
