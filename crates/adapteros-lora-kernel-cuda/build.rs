//! Links libaoscuda.so, built by `python adapter-os_b200/build.py` (nvcc for
//! sm_100a, CUDA runtime linked statically).  AOS_CUDA_LIB_DIR names the
//! directory that holds it; the run-time search path is set to the same
//! directory so the backend loads without LD_LIBRARY_PATH.
fn main() {
    println!("cargo:rerun-if-env-changed=AOS_CUDA_LIB_DIR");
    let dir = std::env::var("AOS_CUDA_LIB_DIR")
        .expect("set AOS_CUDA_LIB_DIR to the directory that holds libaoscuda.so");
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=aoscuda");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
}
