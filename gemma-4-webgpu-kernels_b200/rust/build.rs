// build.rs of the reference crate (rust/build.rs) with the CUDA backend enabled.
//
// libgq.so is the C ABI of include/gq.h, built by nvcc for sm_100a through the
// package Makefile (every kernel of csrc/ plus the ABI, CUDA runtime linked
// statically). This script runs that build and tells cargo where the library is.
// GQ_DIR points at the gemma-4-webgpu-kernels_b200 directory of this repository.
fn main() {
    let gq = std::env::var("GQ_DIR").unwrap_or_else(|_| "../gemma-4-webgpu-kernels_b200".into());
    let status = std::process::Command::new("make")
        .args(["-C", &gq])
        .status()
        .expect("running make for libgq");
    assert!(status.success(), "building libgq.so failed");
    println!("cargo:rustc-link-search=native={gq}/gq");
    println!("cargo:rustc-link-lib=dylib=gq");
    // the shared library is found at run time next to where it was built
    println!("cargo:rustc-link-arg=-Wl,-rpath,{gq}/gq");
    println!("cargo:rerun-if-changed={gq}/csrc");
    println!("cargo:rerun-if-changed={gq}/../include/gq.h");
    println!("cargo:rerun-if-env-changed=GQ_DIR");
}
