//! Links libunltd_gpu.so. The library is built by
//! `python unltd-inference_b200/build.py` into `unltd-inference_b200/lib/`;
//! set UNLTD_GPU_LIB_DIR to another directory that holds it if needed.
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = match env::var("UNLTD_GPU_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => {
            let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").expect("CARGO_MANIFEST_DIR"));
            manifest.join("../../unltd-inference_b200/lib")
        }
    };
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=unltd_gpu");
    println!("cargo:rerun-if-env-changed=UNLTD_GPU_LIB_DIR");
}
