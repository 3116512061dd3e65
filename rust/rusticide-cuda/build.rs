//! Links librusticide_cuda.so. The library is built by the CUDA side of the
//! project (`python rusticide_b200/build.py`, nvcc for sm_100a); point
//! RUSTICIDE_CUDA_LIB_DIR at the directory that holds it.

fn main() {
    println!("cargo:rerun-if-env-changed=RUSTICIDE_CUDA_LIB_DIR");
    if let Ok(dir) = std::env::var("RUSTICIDE_CUDA_LIB_DIR") {
        println!("cargo:rustc-link-search=native={dir}");
    }
    println!("cargo:rustc-link-lib=dylib=rusticide_cuda");
}
