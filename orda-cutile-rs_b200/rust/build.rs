//! Build script for the crate's `cuda` feature bound to the B200 library:
//! links `liborda_b200.so` (built by `make -C orda-cutile-rs_b200`). The
//! directory holding it comes from `ORDA_B200_LIB_DIR`, else the
//! `orda-cutile-rs_b200` directory next to the crate. Without the `cuda`
//! feature nothing is linked and the crate stays CPU-only.
use std::env;
use std::path::PathBuf;

fn main() {
    println!("cargo:rerun-if-env-changed=ORDA_B200_LIB_DIR");
    if env::var_os("CARGO_FEATURE_CUDA").is_none() {
        return;
    }
    let dir = match env::var("ORDA_B200_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => {
            let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").expect("CARGO_MANIFEST_DIR"));
            manifest.join("..").join("orda-cutile-rs_b200")
        }
    };
    let lib = dir.join("liborda_b200.so");
    if !lib.exists() {
        panic!("{} not found: build it with `make -C orda-cutile-rs_b200` or set ORDA_B200_LIB_DIR", lib.display());
    }
    println!("cargo:rerun-if-changed={}", lib.display());
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=orda_b200");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
