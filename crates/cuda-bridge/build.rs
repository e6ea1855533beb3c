// Links librustane_cuda.so, built by `python -m rustane_b200.build`
// (rustane_b200/librustane_cuda.so).  RUSTANE_CUDA_LIB_DIR names the directory
// that holds it; the loader must find it at run time too (rpath or LD_LIBRARY_PATH).
fn main() {
    let dir = std::env::var("RUSTANE_CUDA_LIB_DIR")
        .expect("set RUSTANE_CUDA_LIB_DIR to the directory holding librustane_cuda.so");
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=rustane_cuda");
    println!("cargo:rerun-if-env-changed=RUSTANE_CUDA_LIB_DIR");
}
