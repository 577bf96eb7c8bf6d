//! Links `libs1c.so`, which `python -m sys1rust_b200.build` (nvcc, sm_100a) writes into the
//! `sys1rust_b200/` folder of the libs1c repository. `S1C_LIB_DIR` names that folder (or wherever
//! the library was installed); the build stops with a message when it is unset.
use std::path::PathBuf;

fn main() {
    println!("cargo:rerun-if-env-changed=S1C_LIB_DIR");
    let dir = match std::env::var("S1C_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => panic!("set S1C_LIB_DIR to the folder that holds libs1c.so (built by `python -m sys1rust_b200.build`)"),
    };
    if !dir.join("libs1c.so").is_file() {
        panic!("{} has no libs1c.so", dir.display());
    }
    println!("cargo:rerun-if-changed={}", dir.join("libs1c.so").display());
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=s1c");
    // the CUDA runtime that libs1c links against
    let cuda = std::env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into());
    println!("cargo:rustc-link-search=native={cuda}/lib64");
    println!("cargo:rustc-link-lib=dylib=cudart");
    // binaries find libs1c.so where it was built, without LD_LIBRARY_PATH
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
