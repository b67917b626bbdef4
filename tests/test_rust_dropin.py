"""The Rust drop-in (rust/): its FFI matches include/kernrt_cuda.h, and its
patch applies to a KernRT checkout.

No Rust toolchain exists here, so the Rust side cannot be compiled; these
checks pin what a compiler would: every `fn kernrt_cuda_*` the `extern "C"`
block of rust/src/backends/cuda.rs declares exists in the header with the same
arity and the C types its Rust types stand for, the `#[repr(C)]` window struct
matches `kernrt_window`, and rust/cuda.patch is what rust/make_patch.py writes
for the reference checkout and applies to it (`git apply --check`, on a copy).
"""
import os
import re
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kernrt_cuda.h")
CUDA_RS = os.path.join(ROOT, "rust", "src", "backends", "cuda.rs")
PATCH = os.path.join(ROOT, "rust", "cuda.patch")
REFERENCE = os.environ.get("KERNRT_REFERENCE", "/root/reference")

# C parameter / return type -> the Rust type that binds it
C_TO_RUST = {
    "kernrt_cuda_ctx *": "*mut Ctx",
    "kernrt_cuda_ctx **": "*mut *mut Ctx",
    "kernrt_buf": "u64",
    "kernrt_mat": "u64",
    "uint64_t": "u64",
    "size_t": "usize",
    "int": "c_int",
    "float": "f32",
    "const void *": "*const c_void",
    "const float *": "*const f32",
    "float *": "*mut f32",
    "uint64_t *": "*mut u64",
    "kernrt_buf *": "*mut u64",
    "kernrt_mat *": "*mut u64",
    "const uint64_t *": "*const u64",
    "const kernrt_window *": "*const KernrtWindow",
    "const char *": "*const c_char",
}


def _norm_c_param(p: str) -> str:
    """'const float *x' -> 'const float *', 'kernrt_cuda_ctx **out' -> 'kernrt_cuda_ctx **'."""
    toks = " ".join(p.replace("*", " * ").split()).split(" ")
    if len(toks) > 1 and re.fullmatch(r"[A-Za-z_]\w*", toks[-1]):
        toks = toks[:-1]  # the parameter name
    stars = toks.count("*")
    base = " ".join(t for t in toks if t != "*")
    return base + (" " + "*" * stars if stars else "")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for ret, name, params in re.findall(r"(int|const char \*)\s*(kernrt_cuda_\w+)\s*\(([^)]*)\)\s*;", text):
        ps = [] if params.strip() in ("", "void") else [_norm_c_param(p) for p in params.split(",")]
        out[name] = (ret.strip(), ps)
    return out


def rust_functions():
    text = open(CUDA_RS).read()
    block = re.search(r'unsafe extern "C" \{(.*?)\n\}', text, flags=re.S).group(1)
    out = {}
    for name, params, ret in re.findall(r"fn (kernrt_cuda_\w+)\(([^)]*)\)\s*->\s*([^;]+);", block, flags=re.S):
        ps = [" ".join(p.split(":", 1)[1].split()) for p in params.split(",") if p.strip()]
        out[name] = (" ".join(ret.split()), ps)
    return out


def test_rust_ffi_matches_the_header():
    hdr, rs = header_functions(), rust_functions()
    assert len(rs) >= 25, sorted(rs)
    for name, (ret, params) in rs.items():
        assert name in hdr, f"{name} is not declared in include/kernrt_cuda.h"
        c_ret, c_params = hdr[name]
        assert ret == C_TO_RUST[c_ret], f"{name}: returns {ret}, the header {c_ret}"
        assert len(params) == len(c_params), f"{name}: {len(params)} parameters, the header has {len(c_params)}"
        for i, (r, c) in enumerate(zip(params, c_params)):
            assert c in C_TO_RUST, f"{name}: no Rust binding rule for C type {c!r}"
            assert r == C_TO_RUST[c], f"{name} parameter {i}: Rust {r!r} for C {c!r}"


def test_rust_window_and_kinds_match_the_header():
    text = open(CUDA_RS).read()
    fields = re.search(r"struct KernrtWindow \{(.*?)\}", text, flags=re.S).group(1)
    rust_fields = [(n, t) for n, t in re.findall(r"(\w+): (\w+)", fields)]
    hdr = open(HEADER).read()
    c_fields = re.search(r"typedef struct \{([^}]*)\} kernrt_window;", hdr, flags=re.S).group(1)
    names = re.findall(r"uint64_t ([\w, ]+);", c_fields)[0].replace(" ", "").split(",")
    assert rust_fields == [(n, "u64") for n in names]
    enum = dict(re.findall(r"(KERNRT_(?:F32|BF16|Q8_0X4|Q8_0)) = (\d+)", hdr))
    for rust_name, c_name in [("KIND_F32", "KERNRT_F32"), ("KIND_BF16", "KERNRT_BF16"), ("KIND_Q8_0", "KERNRT_Q8_0")]:
        m = re.search(rf"const {rust_name}: c_int = (\d+);", text)
        assert m and m.group(1) == enum[c_name], rust_name


def test_rust_ffi_symbols_are_exported():
    """Every function the Rust file binds is exported by the built library
    (symbol table only; nothing is called)."""
    lib = os.path.join(ROOT, "kernrt_b200", "_lib", "libkernrt_cuda.so")
    if not os.path.exists(lib):
        pytest.skip("library not built")
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True).stdout
    exported = set(line.split()[-1] for line in out.splitlines() if line.strip())
    missing = sorted(set(rust_functions()) - exported)
    assert not missing, missing


@pytest.mark.skipif(not os.path.isdir(REFERENCE), reason="no KernRT checkout here")
def test_patch_is_current_and_applies(tmp_path):
    sys.path.insert(0, os.path.join(ROOT, "rust"))
    try:
        import make_patch
    finally:
        sys.path.pop(0)
    assert open(PATCH).read() == make_patch.patch_text(REFERENCE), "rust/cuda.patch is stale: rerun make_patch.py"
    if shutil.which("git") is None:
        pytest.skip("no git")
    work = tmp_path / "kernrt"
    work.mkdir()
    for rel in ("Cargo.toml", "src", "tests"):
        src = os.path.join(REFERENCE, rel)
        (shutil.copytree if os.path.isdir(src) else shutil.copy)(src, work / rel)
    r = subprocess.run(["git", "apply", "--check", PATCH], cwd=work, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    subprocess.run(["git", "apply", PATCH], cwd=work, check=True)
    mod = (work / "src" / "backends" / "mod.rs").read_text()
    assert '"cuda" | "nvidia" => cuda::Cuda::new()' in mod and "pub mod cuda;" in mod
    assert (work / "src" / "backends" / "cuda.rs").read_text() == open(CUDA_RS).read()
    assert "cuda = []" in (work / "Cargo.toml").read_text()
    tests = (work / "tests" / "backends.rs").read_text()
    assert "fn cuda_matches_the_scalar_oracle()" in tests
    assert '#[cfg(not(feature = "cuda"))]\n#[test]\nfn unknown_backend_is_an_error()' in tests
