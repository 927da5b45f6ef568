//! Links libtrit_cuda.so. TRIT_CUDA_LIB_DIR names the folder that holds it
//! (default: the repository's trit_b200/ folder, where `make -C
//! trit_b200/csrc` writes it).
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = env::var("TRIT_CUDA_LIB_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../trit_b200")
    });
    println!("cargo:rerun-if-env-changed=TRIT_CUDA_LIB_DIR");
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=trit_cuda");
}
