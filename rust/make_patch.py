#!/usr/bin/env python3
"""Write rust/cuda.patch: the `cuda` backend as a patch to a KernRT checkout.

    python rust/make_patch.py <kernrt-checkout> [out.patch]

The patch adds the two files of this directory (build.rs at the crate root,
src/backends/cuda.rs) and makes the registration edits the backend needs, the
shape of the `metal` feature:

  Cargo.toml          a `cuda = []` feature beside `metal` (Cargo.toml:40-42);
  src/backends/mod.rs `pub mod cuda` under the feature (beside mod.rs:35-38),
                      "cuda" in `available()` (mod.rs:216-225) and a
                      `"cuda" | "nvidia"` arm in `open` (mod.rs:228-244);
  tests/backends.rs   `unknown_backend_is_an_error` (which uses "cuda" as its
                      unknown name, :197-204) only without the feature, and the
                      device parity tests on the model of
                      `metal_matches_the_scalar_oracle` (:333-380).

Each edit is anchored on text of the checkout and fails loudly if that text
is missing or appears more than once.  Apply with `git apply cuda.patch` in
the checkout, then build with `KERNRT_CUDA_DIR=<this repository> cargo test
--features cuda`.
"""
from __future__ import annotations

import difflib
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

CARGO_ANCHOR = 'metal = ["dep:metal"]\n'
CARGO_ADD = '''
# The NVIDIA B200 (sm_100a) backend. Off by default: it needs nvcc and a CUDA
# driver; build.rs builds libkernrt_cuda.so in the checkout KERNRT_CUDA_DIR names.
cuda = []
'''

MOD_DOC_OLD = "//! Selection is [`from_env`] (`KERNRT_BACKEND=cpu|metal|reference`) or [`open`].\n"
MOD_DOC_NEW = "//! Selection is [`from_env`] (`KERNRT_BACKEND=cpu|metal|cuda|reference`) or [`open`].\n"
MOD_DECL_ANCHOR = "pub mod cpu;\n"
MOD_DECL_ADD = '#[cfg(feature = "cuda")]\npub mod cuda;\n'
AVAILABLE_OLD = '''    #[cfg(not(all(target_os = "macos", feature = "metal")))]
    {
        &["cpu", "reference"]
    }
'''
AVAILABLE_NEW = '''    #[cfg(all(not(all(target_os = "macos", feature = "metal")), feature = "cuda"))]
    {
        &["cpu", "cuda", "reference"]
    }
    #[cfg(not(any(all(target_os = "macos", feature = "metal"), feature = "cuda")))]
    {
        &["cpu", "reference"]
    }
'''
OPEN_ANCHOR = '''        other => Err(BackendError {
            requested: other.to_string(),
            detail: None,
        }),
'''
OPEN_ADD = '''        #[cfg(feature = "cuda")]
        "cuda" | "nvidia" => cuda::Cuda::new()
            .map(|b| Box::new(b) as Box<dyn Backend>)
            .map_err(|detail| BackendError {
                requested: name.to_string(),
                detail: Some(detail),
            }),
'''

TEST_GATE_OLD = "#[test]\nfn unknown_backend_is_an_error() {\n"
TEST_GATE_NEW = ('// "cuda" is the unknown name here; with the feature it resolves.\n'
                 '#[cfg(not(feature = "cuda"))]\n#[test]\nfn unknown_backend_is_an_error() {\n')
TEST_ADD = '''
/// The CUDA backend, when compiled in and a device is present.
///
/// The standard the Metal backend meets: decode and batched prefill match the
/// scalar oracle (1e-3 and the same argmax; 5e-2 for the quantized storages,
/// where the oracle quantizes activations too), and so do shared-prefix leaves.
#[cfg(feature = "cuda")]
#[test]
fn cuda_matches_the_scalar_oracle() {
    if let Err(error) = kernrt::backends::open("cuda") {
        // "no device" is a skip; anything else is a broken build or kernel.
        assert!(
            error.to_string().contains("no CUDA device"),
            "CUDA is present but failed to start: {error}"
        );
        eprintln!("skipping: no CUDA device available");
        return;
    }
    for (storage, tol) in [("f32", 1e-3f32), ("bf16", 1e-3), ("q8_0", 5e-2), ("q8_0x4", 5e-2)] {
        let build = |name: &str| {
            Llama::with_backend(
                config(),
                weights_at(&config(), storage),
                kernrt::backends::open(name).unwrap(),
            )
        };
        let prompt: Vec<usize> = vec![5, 11, 2, 30, 7, 7, 19, 1, 24];
        let mut gpu = build("cuda");
        let mut oracle = build("reference");
        let mut want = Vec::new();
        for (pos, &token) in prompt.iter().enumerate() {
            let a = gpu.forward(token, pos).to_vec();
            want = oracle.forward(token, pos).to_vec();
            let diff = max_diff(&a, &want);
            assert!(diff <= tol, "{storage}: decode differs at {pos} by {diff}");
            assert_eq!(argmax(&a), argmax(&want), "{storage}: different token at {pos}");
        }
        let got = build("cuda").prefill(&prompt, 0).to_vec();
        let diff = max_diff(&got, &want);
        assert!(diff <= tol, "{storage}: prefill differs from decode by {diff}");
        assert_eq!(argmax(&got), argmax(&want), "{storage}: prefill picked a different token");

        let prefix = vec![4, 9, 14];
        let suffixes: [&[usize]; 3] = [&[20, 6], &[12, 12, 12, 12], &[31]];
        let a = build("cuda").prefill_shared(&prefix, &suffixes);
        let b = build("reference").prefill_shared(&prefix, &suffixes);
        assert_eq!(a.len(), b.len());
        for (i, (x, y)) in a.iter().zip(&b).enumerate() {
            let diff = max_diff(x, y);
            assert!(diff <= tol, "{storage}: shared-prefix leaf {i} differs by {diff}");
        }
    }
}

/// `open("cuda")` is the switch: with the feature, the name resolves (or says
/// why it cannot) and `available()` lists it.
#[cfg(feature = "cuda")]
#[test]
fn cuda_is_selected_by_name() {
    assert!(kernrt::backends::available().contains(&"cuda"));
    match kernrt::backends::open("cuda") {
        Ok(backend) => assert_eq!(backend.name(), "cuda"),
        Err(error) => {
            assert_eq!(error.requested, "cuda");
            assert!(error.to_string().contains("no CUDA device"), "{error}");
        }
    }
}
'''


def replace_once(text: str, old: str, new: str, where: str) -> str:
    n = text.count(old)
    if n != 1:
        raise SystemExit(f"{where}: expected the anchor once, found it {n} times:\n{old}")
    return text.replace(old, new)


def edits(ref: str) -> dict:
    """path -> (old text, new text) for every file the patch touches."""
    def read(rel):
        with open(os.path.join(ref, rel)) as fh:
            return fh.read()

    out = {}
    cargo = read("Cargo.toml")
    out["Cargo.toml"] = (cargo, replace_once(cargo, CARGO_ANCHOR, CARGO_ANCHOR + CARGO_ADD, "Cargo.toml"))
    mod = read("src/backends/mod.rs")
    new = replace_once(mod, MOD_DOC_OLD, MOD_DOC_NEW, "mod.rs doc")
    new = replace_once(new, MOD_DECL_ANCHOR, MOD_DECL_ANCHOR + MOD_DECL_ADD, "mod.rs modules")
    new = replace_once(new, AVAILABLE_OLD, AVAILABLE_NEW, "mod.rs available()")
    new = replace_once(new, OPEN_ANCHOR, OPEN_ADD + OPEN_ANCHOR, "mod.rs open()")
    out["src/backends/mod.rs"] = (mod, new)
    tests = read("tests/backends.rs")
    new = replace_once(tests, TEST_GATE_OLD, TEST_GATE_NEW, "tests/backends.rs gate")
    out["tests/backends.rs"] = (tests, new.rstrip("\n") + "\n" + TEST_ADD)
    for rel, src in (("build.rs", "build.rs"), ("src/backends/cuda.rs", "src/backends/cuda.rs")):
        if os.path.exists(os.path.join(ref, rel)):
            raise SystemExit(f"{rel} already exists in {ref}")
        with open(os.path.join(HERE, src)) as fh:
            out[rel] = (None, fh.read())
    return out


def patch_text(ref: str) -> str:
    parts = []
    for rel, (old, new) in edits(ref).items():
        if old is None:
            lines = new.splitlines(keepends=True)
            parts.append(f"diff --git a/{rel} b/{rel}\nnew file mode 100644\n--- /dev/null\n+++ b/{rel}\n"
                         f"@@ -0,0 +1,{len(lines)} @@\n")
            parts.extend("+" + ln for ln in lines)
            continue
        parts.append(f"diff --git a/{rel} b/{rel}\n")
        parts.extend(difflib.unified_diff(old.splitlines(keepends=True), new.splitlines(keepends=True),
                                          fromfile=f"a/{rel}", tofile=f"b/{rel}", n=3))
    return "".join(parts)


def main() -> None:
    if len(sys.argv) < 2:
        raise SystemExit(__doc__)
    out = sys.argv[2] if len(sys.argv) > 2 else os.path.join(HERE, "cuda.patch")
    with open(out, "w") as fh:
        fh.write(patch_text(sys.argv[1]))
    print(f"wrote {out}")


if __name__ == "__main__":
    main()
