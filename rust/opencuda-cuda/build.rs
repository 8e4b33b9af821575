//! Builds libopencuda_cuda.so (nvcc, sm_100a, static CUDA runtime) with the
//! library's own Makefile and links it.  OPENCUDA_B200_DIR names the
//! directory that holds the Makefile (the repository's open-cuda_b200/);
//! the default is ../../open-cuda_b200 relative to this crate.
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let dir = match std::env::var("OPENCUDA_B200_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(env!("CARGO_MANIFEST_DIR")).join("../../open-cuda_b200"),
    };
    let status = Command::new("make")
        .arg("-C")
        .arg(&dir)
        .status()
        .expect("running make for libopencuda_cuda.so");
    assert!(status.success(), "building libopencuda_cuda.so failed (needs nvcc 12.8 or newer for sm_100a)");
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=opencuda_cuda");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
    println!("cargo:rerun-if-changed={}", dir.join("csrc").display());
    println!("cargo:rerun-if-env-changed=OPENCUDA_B200_DIR");
}
