// Link libglypr_cuda.so: GLYPR_CUDA_LIB_DIR names the directory holding it (by default the
// package directory of this repository, where glypr_b200/build.py writes it).  The library
// links the CUDA runtime statically, so only the NVIDIA driver is needed at run time.
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = env::var("GLYPR_CUDA_LIB_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("..").join("..")
    });
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=glypr_cuda");
    println!("cargo:rerun-if-env-changed=GLYPR_CUDA_LIB_DIR");
}
