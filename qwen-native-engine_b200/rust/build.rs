//! Links libqne.so: from QNE_LIB_DIR if set, else the in-tree build next to the Python package
//! (qwen-native-engine_b200/qne/_lib), and records that directory as the run-time search path.
use std::path::PathBuf;

fn main() {
    let dir = match std::env::var("QNE_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").unwrap()).join("../qne/_lib"),
    };
    let dir = dir.canonicalize().unwrap_or(dir);
    println!("cargo:rerun-if-env-changed=QNE_LIB_DIR");
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=qne");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
