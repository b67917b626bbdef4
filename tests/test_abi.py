"""The C-ABI library loads and exports every entry point include/kernrt_cuda.h
declares (no GPU needed; no compute calls)."""
import ctypes
import os
import re

import pytest

import kernrt_b200

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "kernrt_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kernrt_cuda_\w+)\s*\(", text)))


def test_header_declares_the_trait_surface():
    names = declared_functions()
    # Every Backend trait op on the hot path has an entry point (mod.rs:264-404).
    for op in ["create", "destroy", "name", "storage", "prepare_embedding", "alloc", "upload", "read",
               "embed", "copy", "rms_norm", "qk_norm", "rope", "add_in_place", "mul", "conv_prefill",
               "conv_decode", "silu_mul"]:
        assert f"kernrt_cuda_{op}" in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(kernrt_b200.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_python_binding_covers_the_header():
    assert set(declared_functions()) == set(kernrt_b200.SIGNATURES)


def test_chain_struct_matches_header_field_order():
    text = open(HEADER).read()
    body = text[text.index("typedef struct {", text.index("the fused layer-op chain")):]
    body = body[:body.index("} kernrt_chain_args;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl or decl.startswith("typedef"):
            decl = decl.replace("typedef struct {", "").strip()
            if not decl:
                continue
        names = decl.split(None, 1)[1]
        fields += [n.strip() for n in names.split(",")]
    assert fields == [n for n, _ in kernrt_b200.ChainArgs._fields_]


def test_device_count_never_fails():
    assert kernrt_b200.device_count() >= 0


def test_missing_device_is_a_specific_error():
    """The Metal backend's contract (tests/backends.rs:335-348): a machine without
    the device yields a distinguishable error, never a silent fallback."""
    if kernrt_b200.device_count() > 0:
        pytest.skip("a CUDA device is present")
    with pytest.raises(kernrt_b200.KernrtCudaError) as err:
        kernrt_b200.CudaBackend()
    assert err.value.code == kernrt_b200.E_NO_DEVICE
    assert "no CUDA device" in str(err.value)


def test_unknown_backend_name_is_an_error():
    """tests/backends.rs:197-204: `open` fails loudly on unknown names."""
    with pytest.raises(kernrt_b200.KernrtCudaError) as err:
        kernrt_b200.open_backend("metal")
    assert "available" in str(err.value)


def test_null_context_is_rejected():
    lib = kernrt_b200.load()
    assert lib.kernrt_cuda_synchronize(None) == kernrt_b200.E_INVALID
    assert "null" in kernrt_b200.last_error()
