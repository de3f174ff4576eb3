//! Builds libst_b200.so (nvcc, sm_100a) from the scratchtape-b200 tree and
//! links it.  SCRATCHTAPE_B200_DIR points at that tree (default: two levels
//! up from this crate, where it lives in the repository).
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let root = std::env::var("SCRATCHTAPE_B200_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").unwrap()).join("..").join("..")
    });
    // scratchtape_b200/build.py runs nvcc -gencode arch=compute_100a,code=sm_100a per .cu
    // file and links the shared library with the static CUDA runtime
    let status = Command::new("python3")
        .arg(root.join("scratchtape_b200").join("build.py"))
        .current_dir(&root)
        .status()
        .expect("running scratchtape_b200/build.py (needs python3 and nvcc)");
    assert!(status.success(), "building libst_b200.so failed");
    let lib_dir = root.join("scratchtape_b200");
    println!("cargo:rustc-link-search=native={}", lib_dir.display());
    println!("cargo:rustc-link-lib=dylib=st_b200");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", lib_dir.display());
    println!("cargo:rerun-if-changed={}", root.join("scratchtape_b200").join("csrc").display());
    println!("cargo:rerun-if-changed={}", root.join("include").join("st_b200.h").display());
    println!("cargo:rerun-if-env-changed=SCRATCHTAPE_B200_DIR");
}
