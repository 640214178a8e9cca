//! Links libdiffrast_cuda.so. Set DIFFRAST_CUDA_LIB_DIR to the directory that
//! holds it (the in-tree build puts it in differentiable-rasterizer_b200/diffrast/);
//! the same directory is recorded as an rpath so the loader finds it at run time.

fn main() {
    println!("cargo:rerun-if-env-changed=DIFFRAST_CUDA_LIB_DIR");
    if let Ok(dir) = std::env::var("DIFFRAST_CUDA_LIB_DIR") {
        println!("cargo:rustc-link-search=native={dir}");
        println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
    }
    println!("cargo:rustc-link-lib=dylib=diffrast_cuda");
}
