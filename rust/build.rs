//! KernRT's build script for the `cuda` feature (KernRT has no build.rs of its
//! own; Cargo runs one found at the crate root).  Without the feature it does
//! nothing.  With it, it builds libkernrt_cuda.so with nvcc (the library's
//! Makefile, sm_100a) in the kernrt-b200 checkout named by KERNRT_CUDA_DIR and
//! links it, with an rpath so tests and examples find it at run time.

fn main() {
    println!("cargo:rerun-if-env-changed=KERNRT_CUDA_DIR");
    if std::env::var_os("CARGO_FEATURE_CUDA").is_none() {
        return;
    }
    let dir = std::env::var("KERNRT_CUDA_DIR")
        .expect("the cuda feature needs KERNRT_CUDA_DIR: the path of a kernrt-b200 checkout");
    let status = std::process::Command::new("make")
        .args(["-C", &format!("{dir}/kernrt_b200/csrc")])
        .status()
        .expect("running make for libkernrt_cuda.so (needs nvcc on PATH or NVCC=...)");
    assert!(status.success(), "building libkernrt_cuda.so failed");
    println!("cargo:rustc-link-search=native={dir}/kernrt_b200/_lib");
    println!("cargo:rustc-link-lib=dylib=kernrt_cuda");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}/kernrt_b200/_lib");
    println!("cargo:rerun-if-changed={dir}/kernrt_b200/csrc");
    println!("cargo:rerun-if-changed={dir}/include/kernrt_cuda.h");
}
