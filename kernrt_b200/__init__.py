"""kernrt_b200 — the B200 (sm_100a) `cuda` backend for KernRT's per-row layer ops.

The product is the C-ABI library ``_lib/libkernrt_cuda.so`` (declared in
``include/kernrt_cuda.h``).  This package loads it through ctypes and exposes
:class:`CudaBackend`, a Python mirror of KernRT's ``Backend`` trait
(src/backends/mod.rs:264-404): same method names, same argument meaning,
handles instead of slices, ``read`` as the only barrier.  Failures raise
:class:`KernrtCudaError`, where the Rust reference panics.

There is no CPU fallback: if the library is missing, :func:`load` raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "_lib", "libkernrt_cuda.so")
HEADER = os.path.join(ROOT, "include", "kernrt_cuda.h")

F32, BF16, Q8_0, Q8_0X4 = 0, 1, 2, 3
KIND_NAMES = {F32: "f32", BF16: "bf16", Q8_0: "q8_0", Q8_0X4: "q8_0x4"}
E_NO_DEVICE, E_INVALID, E_CUDA, E_DEVICE, E_STATE = 1, 2, 3, 4, 5

_lib = None


class KernrtCudaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def build(force: bool = False) -> str:
    """Compile the sm_100a library in-tree (nvcc; no GPU needed)."""
    args = ["make", "-s", "-C", os.path.join(HERE, "csrc")]
    if force:
        subprocess.run(args + ["clean"], check=True)
    subprocess.run(args, check=True)
    return LIB_PATH


Buf = C.c_uint64
SZ = C.c_size_t
P = C.c_void_p


class ChainArgs(C.Structure):
    """Mirror of ``kernrt_chain_args`` (include/kernrt_cuda.h)."""

    _fields_ = [
        ("rows", SZ), ("dim", SZ), ("q_dim", SZ), ("kv_dim", SZ), ("hidden", SZ), ("head_size", SZ),
        ("eps", C.c_float), ("theta", C.c_float), ("final_eps", C.c_float), ("interleaved", C.c_int),
        ("tokens", Buf), ("positions", Buf), ("x", Buf), ("xb", Buf), ("w_att", Buf),
        ("q", Buf), ("k", Buf), ("w_q", Buf), ("w_k", Buf), ("gate", Buf), ("up", Buf),
        ("resid", Buf), ("w_final", Buf), ("codes", Buf), ("scales", Buf), ("scales_f16", Buf),
    ]


class Window(C.Structure):
    """Mirror of ``kernrt_window``: one query row's causal window."""

    _fields_ = [("att_start", C.c_uint64), ("slot", C.c_uint64), ("shared_start", C.c_uint64),
                ("shared_end", C.c_uint64)]


class StTensor(C.Structure):
    """Mirror of ``kernrt_st_tensor``: one tensor's entry in a safetensors file."""

    _fields_ = [("dtype", C.c_int), ("rank", C.c_int), ("shape", C.c_uint64 * 8),
                ("file_offset", C.c_uint64), ("bytes", C.c_uint64)]


class ChainHostArgs(C.Structure):
    """Mirror of ``kernrt_chain_host_args`` (include/kernrt_cuda.h)."""

    _fields_ = [
        ("rows", SZ), ("dim", SZ), ("q_dim", SZ), ("kv_dim", SZ), ("hidden", SZ), ("head_size", SZ),
        ("eps", C.c_float), ("theta", C.c_float), ("final_eps", C.c_float), ("interleaved", C.c_int),
        ("chunk_rows", SZ),
        ("tokens", P), ("positions", P), ("x_in", P), ("q_in", P), ("k_in", P), ("gate_in", P),
        ("up", P), ("resid", P), ("x_out", P), ("xb_out", P), ("q_out", P), ("k_out", P),
        ("gate_out", P), ("codes", P), ("scales", P), ("scales_f16", P),
        ("w_att", Buf), ("w_q", Buf), ("w_k", Buf), ("w_final", Buf),
    ]


# Every function include/kernrt_cuda.h declares, with its ctypes signature.
SIGNATURES = {
    "kernrt_cuda_last_error": (C.c_char_p, []),
    "kernrt_cuda_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "kernrt_cuda_kernel_launches": (C.c_int, [C.POINTER(C.c_uint64)]),
    "kernrt_cuda_create": (C.c_int, [C.c_int, C.POINTER(P)]),
    "kernrt_cuda_destroy": (C.c_int, [P]),
    "kernrt_cuda_name": (C.c_char_p, [P]),
    "kernrt_cuda_storage": (C.c_char_p, [P]),
    "kernrt_cuda_stream": (C.c_int, [P, C.POINTER(P)]),
    "kernrt_cuda_prepare_embedding": (C.c_int, [P, C.c_int, P, P, SZ, SZ]),
    "kernrt_cuda_alloc": (C.c_int, [P, SZ, C.POINTER(Buf)]),
    "kernrt_cuda_upload": (C.c_int, [P, P, SZ, C.POINTER(Buf)]),
    "kernrt_cuda_read": (C.c_int, [P, Buf, P, SZ]),
    "kernrt_cuda_alloc_bytes": (C.c_int, [P, SZ, C.POINTER(Buf)]),
    "kernrt_cuda_write_bytes": (C.c_int, [P, Buf, SZ, P, SZ]),
    "kernrt_cuda_read_bytes": (C.c_int, [P, Buf, SZ, P, SZ]),
    "kernrt_cuda_device_ptr": (C.c_int, [P, Buf, C.POINTER(P)]),
    "kernrt_cuda_synchronize": (C.c_int, [P]),
    "kernrt_cuda_flush": (C.c_int, [P]),
    "kernrt_cuda_embed": (C.c_int, [P, SZ, Buf, SZ]),
    "kernrt_cuda_copy": (C.c_int, [P, Buf, SZ, Buf, SZ, SZ]),
    "kernrt_cuda_rms_norm": (C.c_int, [P, Buf, Buf, Buf, SZ, SZ, C.c_float]),
    "kernrt_cuda_qk_norm": (C.c_int, [P, Buf, SZ, SZ, SZ, Buf, C.c_float]),
    "kernrt_cuda_rope": (C.c_int, [P, Buf, Buf, SZ, SZ, SZ, P, SZ, SZ, C.c_float, C.c_int]),
    "kernrt_cuda_add_in_place": (C.c_int, [P, Buf, Buf, SZ]),
    "kernrt_cuda_mul": (C.c_int, [P, Buf, SZ, Buf, SZ, Buf, SZ, SZ]),
    "kernrt_cuda_conv_prefill": (C.c_int, [P, Buf, Buf, Buf, SZ, SZ, SZ]),
    "kernrt_cuda_conv_decode": (C.c_int, [P, Buf, Buf, Buf, Buf, SZ, SZ]),
    "kernrt_cuda_silu_mul": (C.c_int, [P, Buf, Buf, SZ]),
    "kernrt_cuda_quantize_q8_0": (C.c_int, [P, Buf, SZ, SZ, Buf, Buf, Buf]),
    "kernrt_cuda_rms_norm_q8_0": (C.c_int, [P, Buf, Buf, SZ, SZ, C.c_float, Buf, Buf, Buf]),
    "kernrt_cuda_rope_prepare": (C.c_int, [P, C.c_float, SZ, SZ]),
    "kernrt_cuda_layer_chain": (C.c_int, [P, C.POINTER(ChainArgs)]),
    "kernrt_cuda_lfm2_conv_block": (C.c_int, [P, Buf, Buf, Buf, Buf, SZ, SZ, SZ]),
    "kernrt_cuda_lfm2_conv_block_halo": (C.c_int, [P, Buf, Buf, Buf, Buf, SZ, SZ, SZ, SZ]),
    "kernrt_cuda_layer_chain_host": (C.c_int, [P, C.POINTER(ChainHostArgs)]),
    "kernrt_cuda_stage_timing": (C.c_int, [P, C.c_int]),
    "kernrt_cuda_stage_times": (C.c_int, [P, C.POINTER(C.c_double), C.POINTER(C.c_uint64)]),
    "kernrt_cuda_prepare_matrix": (C.c_int, [P, C.c_int, P, P, SZ, SZ, C.POINTER(C.c_uint64)]),
    "kernrt_cuda_project": (C.c_int, [P, C.c_uint64, Buf, Buf, SZ]),
    "kernrt_cuda_project_qkv": (C.c_int, [P, C.c_uint64, C.c_uint64, C.c_uint64, Buf, Buf, Buf, Buf, SZ]),
    "kernrt_cuda_project_gate_up": (C.c_int, [P, C.c_uint64, C.c_uint64, Buf, Buf, Buf, SZ]),
    "kernrt_cuda_logits": (C.c_int, [P, C.c_uint64, Buf, Buf]),
    "kernrt_cuda_kv_prepare": (C.c_int, [P, SZ, SZ, SZ]),
    "kernrt_cuda_kv_write": (C.c_int, [P, SZ, P, SZ, Buf, Buf, SZ]),
    "kernrt_cuda_attention": (C.c_int, [P, Buf, Buf, Buf, SZ, C.POINTER(Window), SZ, SZ, SZ, SZ, SZ, SZ]),
    "kernrt_cuda_embed_rows_noalloc": (C.c_int, [C.c_int, C.c_int, P, P, SZ, SZ, P, SZ, P, P]),
    "kernrt_cuda_safetensors_tensor": (C.c_int, [C.c_char_p, C.c_char_p, C.POINTER(StTensor)]),
    "kernrt_cuda_prepare_embedding_file": (C.c_int, [P, C.c_char_p, C.c_char_p, C.c_int]),
    "kernrt_cuda_selftest_wait": (C.c_int, [P, C.c_uint64, C.c_int]),
    "kernrt_cuda_set_exact": (C.c_int, [P, C.c_int]),
}

# safetensors dtypes (kernrt_st_tensor.dtype)
ST_F32, ST_BF16, ST_F16 = 0, 1, 2
ST_DTYPES = {ST_F32: "F32", ST_BF16: "BF16", ST_F16: "F16"}

NOALLOC_MAX_ROWS = 65536


def load() -> C.CDLL:
    """Load the backend library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise KernrtCudaError(E_STATE, f"{LIB_PATH} is not built (run kernrt_b200.build())")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def last_error() -> str:
    return load().kernrt_cuda_last_error().decode()


def _ok(rc: int) -> None:
    if rc != 0:
        raise KernrtCudaError(rc, last_error())


def device_count() -> int:
    n = C.c_int(0)
    _ok(load().kernrt_cuda_device_count(C.byref(n)))
    return n.value


def kernel_launches() -> int:
    """Kernels the library has launched in this process (all devices)."""
    n = C.c_uint64(0)
    _ok(load().kernrt_cuda_kernel_launches(C.byref(n)))
    return n.value


def safetensors_tensor(path: str, name: str) -> dict:
    """One tensor's entry in a safetensors file, read and validated on the host
    as src/formats/safetensors.rs:161-257 does (no device involved): dtype name,
    shape, and the payload's byte range in the file."""
    t = StTensor()
    _ok(load().kernrt_cuda_safetensors_tensor(os.fsencode(path), name.encode(), C.byref(t)))
    return {"dtype": ST_DTYPES[t.dtype], "shape": tuple(t.shape[i] for i in range(min(t.rank, 8))),
            "offset": t.file_offset, "bytes": t.bytes}


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


class CudaBackend:
    """KernRT's ``Backend`` trait over the sm_100a library (one CUDA device)."""

    def __init__(self, device: int = -1):
        self._lib = load()
        ctx = P()
        _ok(self._lib.kernrt_cuda_create(int(device), C.byref(ctx)))
        self._ctx = ctx
        self._lens: dict[int, int] = {}

    # -- lifecycle ----------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_ctx", None):
            self._lib.kernrt_cuda_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- identity (mod.rs:265-269) ----------------------------------------------------
    def name(self) -> str:
        return self._lib.kernrt_cuda_name(self._ctx).decode()

    def storage(self) -> str:
        return self._lib.kernrt_cuda_storage(self._ctx).decode()

    def stream(self) -> int:
        s = P()
        _ok(self._lib.kernrt_cuda_stream(self._ctx, C.byref(s)))
        return s.value or 0

    # -- prepare ---------------------------------------------------------------------
    def prepare_embedding(self, kind: int, data: np.ndarray, scales: np.ndarray | None,
                          vocab: int, dim: int) -> None:
        data = np.ascontiguousarray(data)
        sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.float32)
        _ok(self._lib.kernrt_cuda_prepare_embedding(self._ctx, kind, _ptr(data),
                                                    None if sc is None else _ptr(sc), vocab, dim))
        self._keep = (data, sc)

    def prepare_embedding_file(self, path: str, name: str = "model.embed_tokens.weight",
                               storage: int = 1) -> None:
        """The token embedding straight from a safetensors file (hf.rs:141-191):
        the stored payload goes to the device and is converted there into the
        storage matrix_from_raw picks for ``storage`` (default bf16)."""
        _ok(self._lib.kernrt_cuda_prepare_embedding_file(self._ctx, os.fsencode(path), name.encode(),
                                                         int(storage)))

    def selftest_wait(self, cycles: int, complete: bool) -> None:
        """The kernels' bounded wait run alone: raises KernrtCudaError
        (E_DEVICE, "... timed out") when the phase is left incomplete."""
        _ok(self._lib.kernrt_cuda_selftest_wait(self._ctx, int(cycles), int(bool(complete))))

    # -- buffers ---------------------------------------------------------------------
    def alloc(self, length: int) -> int:
        h = Buf()
        _ok(self._lib.kernrt_cuda_alloc(self._ctx, length, C.byref(h)))
        return h.value

    def alloc_bytes(self, nbytes: int) -> int:
        h = Buf()
        _ok(self._lib.kernrt_cuda_alloc_bytes(self._ctx, nbytes, C.byref(h)))
        return h.value

    def upload(self, data) -> int:
        a = np.ascontiguousarray(data, dtype=np.float32).ravel()
        h = Buf()
        _ok(self._lib.kernrt_cuda_upload(self._ctx, _ptr(a), a.size, C.byref(h)))
        return h.value

    def upload_bytes(self, data: np.ndarray) -> int:
        a = np.ascontiguousarray(data)
        h = self.alloc_bytes(a.nbytes)
        self.write_bytes(h, a)
        return h

    def write_bytes(self, buf: int, data: np.ndarray, byte_offset: int = 0) -> None:
        a = np.ascontiguousarray(data)
        _ok(self._lib.kernrt_cuda_write_bytes(self._ctx, buf, byte_offset, _ptr(a), a.nbytes))

    def write_ptr(self, buf: int, host_ptr: int, nbytes: int, byte_offset: int = 0) -> None:
        _ok(self._lib.kernrt_cuda_write_bytes(self._ctx, buf, byte_offset, host_ptr, nbytes))

    def read(self, src: int, length: int) -> np.ndarray:
        out = np.empty(length, np.float32)
        _ok(self._lib.kernrt_cuda_read(self._ctx, src, _ptr(out), length))
        return out

    def read_into(self, src: int, out: np.ndarray) -> None:
        _ok(self._lib.kernrt_cuda_read_bytes(self._ctx, src, 0, _ptr(out), out.nbytes))

    def read_ptr(self, src: int, host_ptr: int, nbytes: int, byte_offset: int = 0) -> None:
        _ok(self._lib.kernrt_cuda_read_bytes(self._ctx, src, byte_offset, host_ptr, nbytes))

    def read_bytes(self, src: int, nbytes: int, dtype) -> np.ndarray:
        out = np.empty(nbytes // np.dtype(dtype).itemsize, dtype)
        _ok(self._lib.kernrt_cuda_read_bytes(self._ctx, src, 0, _ptr(out), out.nbytes))
        return out

    def device_ptr(self, buf: int) -> int:
        p = P()
        _ok(self._lib.kernrt_cuda_device_ptr(self._ctx, buf, C.byref(p)))
        return p.value or 0

    def synchronize(self) -> None:
        _ok(self._lib.kernrt_cuda_synchronize(self._ctx))

    def flush(self) -> None:
        """Launch deferred work without waiting for it."""
        _ok(self._lib.kernrt_cuda_flush(self._ctx))

    # -- the row ops (mod.rs:284-400) ------------------------------------------------
    def embed(self, token: int, out: int, offset: int) -> None:
        _ok(self._lib.kernrt_cuda_embed(self._ctx, token, out, offset))

    def copy(self, src: int, src_offset: int, dst: int, dst_offset: int, length: int) -> None:
        _ok(self._lib.kernrt_cuda_copy(self._ctx, src, src_offset, dst, dst_offset, length))

    def rms_norm(self, out: int, x: int, weight: int, rows: int, dim: int, eps: float) -> None:
        _ok(self._lib.kernrt_cuda_rms_norm(self._ctx, out, x, weight, rows, dim, eps))

    def qk_norm(self, v: int, rows: int, width: int, head_size: int, weight: int, eps: float) -> None:
        _ok(self._lib.kernrt_cuda_qk_norm(self._ctx, v, rows, width, head_size, weight, eps))

    def rope(self, q: int, k: int, q_width: int, kv_width: int, rows: int, positions,
             head_size: int, theta: float, interleaved: bool) -> None:
        pos = np.ascontiguousarray(positions, dtype=np.uint64)
        _ok(self._lib.kernrt_cuda_rope(self._ctx, q, k, q_width, kv_width, rows, _ptr(pos), pos.size,
                                       head_size, theta, int(bool(interleaved))))

    def add_in_place(self, dst: int, src: int, length: int) -> None:
        _ok(self._lib.kernrt_cuda_add_in_place(self._ctx, dst, src, length))

    def mul(self, out: int, out_off: int, a: int, a_off: int, b: int, b_off: int, length: int) -> None:
        _ok(self._lib.kernrt_cuda_mul(self._ctx, out, out_off, a, a_off, b, b_off, length))

    def conv_prefill(self, out: int, x: int, kernel: int, rows: int, dim: int, k: int) -> None:
        _ok(self._lib.kernrt_cuda_conv_prefill(self._ctx, out, x, kernel, rows, dim, k))

    def conv_decode(self, out: int, x: int, kernel: int, state: int, dim: int, k: int) -> None:
        _ok(self._lib.kernrt_cuda_conv_decode(self._ctx, out, x, kernel, state, dim, k))

    def silu_mul(self, gate: int, up: int, length: int) -> None:
        _ok(self._lib.kernrt_cuda_silu_mul(self._ctx, gate, up, length))

    # -- beyond the trait --------------------------------------------------------------
    def quantize_q8_0(self, x: int, rows: int, dim: int, codes: int, scales: int,
                      scales_f16: int = 0) -> None:
        _ok(self._lib.kernrt_cuda_quantize_q8_0(self._ctx, x, rows, dim, codes, scales, scales_f16))

    def rms_norm_q8_0(self, x: int, weight: int, rows: int, dim: int, eps: float, codes: int,
                      scales: int, scales_f16: int = 0) -> None:
        _ok(self._lib.kernrt_cuda_rms_norm_q8_0(self._ctx, x, weight, rows, dim, eps, codes, scales,
                                                scales_f16))

    def rope_prepare(self, theta: float, head_size: int, max_pos: int) -> None:
        _ok(self._lib.kernrt_cuda_rope_prepare(self._ctx, theta, head_size, max_pos))

    def layer_chain(self, **kw) -> None:
        a = ChainArgs()
        for name, _ in ChainArgs._fields_:
            if name in kw and kw[name] is not None:
                setattr(a, name, kw[name])
        unknown = set(kw) - {n for n, _ in ChainArgs._fields_}
        if unknown:
            raise TypeError(f"unknown chain arguments {sorted(unknown)}")
        _ok(self._lib.kernrt_cuda_layer_chain(self._ctx, C.byref(a)))

    def layer_chain_host(self, **kw) -> None:
        """kernrt_cuda_layer_chain_host: host arrays (numpy, or integer host
        addresses) for the row inputs/outputs, handles for the weights."""
        a = ChainHostArgs()
        names = {n for n, _ in ChainHostArgs._fields_}
        unknown = set(kw) - names
        if unknown:
            raise TypeError(f"unknown chain arguments {sorted(unknown)}")
        keep = []
        for name, ctype in ChainHostArgs._fields_:
            v = kw.get(name)
            if v is None:
                continue
            if ctype is P and isinstance(v, np.ndarray):
                assert v.flags["C_CONTIGUOUS"]
                keep.append(v)
                v = v.ctypes.data
            setattr(a, name, v)
        _ok(self._lib.kernrt_cuda_layer_chain_host(self._ctx, C.byref(a)))

    # the norm stage is k_norm_rows, k_norm_cols, k_norm_small or k_norm_pipe by source, rows and width
    STAGES = ("norm", "stream", "fused")

    def stage_timing(self, enable: bool) -> None:
        _ok(self._lib.kernrt_cuda_stage_timing(self._ctx, int(bool(enable))))

    def stage_times(self) -> dict:
        """{stage: (total device ms, launches)} since stage timing was enabled."""
        ms = (C.c_double * 3)()
        n = (C.c_uint64 * 3)()
        _ok(self._lib.kernrt_cuda_stage_times(self._ctx, ms, n))
        return {k: (ms[i], n[i]) for i, k in enumerate(self.STAGES)}

    # -- contractions (reference.rs:151-159, 259-306, 402-416) ----------------------
    def prepare_matrix(self, kind: int, data: np.ndarray, scales: np.ndarray | None, out_dim: int,
                       in_dim: int) -> int:
        """Uploads W [out_dim, in_dim] in its stored format; returns its handle."""
        data = np.ascontiguousarray(data)
        sc = None if scales is None else np.ascontiguousarray(scales, dtype=np.float32)
        h = C.c_uint64()
        _ok(self._lib.kernrt_cuda_prepare_matrix(self._ctx, kind, _ptr(data), None if sc is None else _ptr(sc),
                                                 out_dim, in_dim, C.byref(h)))
        return h.value

    def set_exact(self, exact: bool) -> None:
        """kernrt_cuda_set_exact: False sends bf16 projections of >= 16 rows to
        the tensor cores and those of 1-4 rows to warp-wide sums (tolerance
        mode); True (the default) keeps them in the reference's order."""
        _ok(self._lib.kernrt_cuda_set_exact(self._ctx, int(bool(exact))))

    def project(self, w: int, x: int, y: int, rows: int) -> None:
        _ok(self._lib.kernrt_cuda_project(self._ctx, w, x, y, rows))

    def project_qkv(self, wq: int, wk: int, wv: int, x: int, q: int, k: int, v: int, rows: int) -> None:
        _ok(self._lib.kernrt_cuda_project_qkv(self._ctx, wq, wk, wv, x, q, k, v, rows))

    def project_gate_up(self, wg: int, wu: int, x: int, gate: int, up: int, rows: int) -> None:
        _ok(self._lib.kernrt_cuda_project_gate_up(self._ctx, wg, wu, x, gate, up, rows))

    def logits(self, w: int, x: int, y: int) -> None:
        _ok(self._lib.kernrt_cuda_logits(self._ctx, w, x, y))

    def kv_prepare(self, n_layers: int, kv_dim: int, seq_len: int) -> None:
        _ok(self._lib.kernrt_cuda_kv_prepare(self._ctx, n_layers, kv_dim, seq_len))

    def kv_write(self, layer: int, slots, k: int, v: int, rows: int) -> None:
        sl = np.ascontiguousarray(slots, dtype=np.uint64)
        _ok(self._lib.kernrt_cuda_kv_write(self._ctx, layer, _ptr(sl), sl.size, k, v, rows))

    def attention(self, q: int, out: int, att: int, layer: int, windows, n_heads: int, kv_mul: int,
                  head_size: int, kv_dim: int, seq_len: int) -> None:
        """windows: sequence of (att_start, slot, shared_start, shared_end)."""
        ws = (Window * max(1, len(windows)))(*[Window(*map(int, w)) for w in windows])
        _ok(self._lib.kernrt_cuda_attention(self._ctx, q, out, att, layer, ws, len(windows), n_heads, kv_mul,
                                            head_size, kv_dim, seq_len))

    def lfm2_conv_block(self, bcx: int, kernel: int, ring: int, cy: int, rows: int, dim: int,
                        k: int) -> None:
        _ok(self._lib.kernrt_cuda_lfm2_conv_block(self._ctx, bcx, kernel, ring, cy, rows, dim, k))

    def lfm2_conv_block_halo(self, bcx: int, kernel: int, ring: int, cy: int, rows: int, dim: int, k: int,
                             halo: int) -> None:
        """kernrt_cuda_lfm2_conv_block_halo: one shard of a sequence, bcx with
        `halo` preceding rows first; ring 0 skips the ring update."""
        _ok(self._lib.kernrt_cuda_lfm2_conv_block_halo(self._ctx, bcx, kernel, ring, cy, rows, dim, k, halo))


def embed_rows_noalloc(device: int, kind: int, table_ptr: int, scales_ptr: int, vocab: int, dim: int,
                       tokens, out_ptr: int, stream: int = 0) -> None:
    """kernrt_cuda_embed_rows_noalloc: gather `tokens` rows of a device table
    into the caller's device rows at `out_ptr` without allocating anything
    (fixed scratch of NOALLOC_MAX_ROWS rows; see include/kernrt_cuda.h)."""
    toks = np.ascontiguousarray(tokens, dtype=np.int32)
    _ok(load().kernrt_cuda_embed_rows_noalloc(device, kind, table_ptr, scales_ptr or None, vocab, dim,
                                              _ptr(toks), toks.size, out_ptr, stream or None))


def open_backend(name: str = "cuda", device: int = -1) -> CudaBackend:
    """``backends::open`` for this package's one backend (mod.rs:228-244)."""
    if name not in ("cuda", "nvidia"):
        raise KernrtCudaError(E_INVALID, f'unknown backend "{name}"; available: cuda')
    return CudaBackend(device)
