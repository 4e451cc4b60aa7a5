//! Links libqora_cuda.so, which the package's own build step compiles with nvcc
//! (`python -c "import __graft_entry__ as g; g.build()"` at the repository root). Its
//! directory comes from QORA_CUDA_LIB_DIR, else the package directory two levels up
//! (qora-llm_b200/, where the build step writes the library).
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = match env::var("QORA_CUDA_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(env::var("CARGO_MANIFEST_DIR").expect("cargo sets CARGO_MANIFEST_DIR")).join("../.."),
    };
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=qora_cuda");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
    println!("cargo:rerun-if-env-changed=QORA_CUDA_LIB_DIR");
}
