//! build.rs for the gpt-sovits-rs crate: builds libgsvdec.so (sm_100a) with
//! the repository's nvcc recipe and links it.
//!
//! Not compiled here: this repository's build image has no Rust toolchain.
//! The nvcc side is `python gpt-sovits-rs_b200/build.py`, which compiles every
//! csrc/*.cu with `-gencode arch=compute_100a,code=sm_100a` into
//! gpt-sovits-rs_b200/_build/libgsvdec.so.

use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let root = PathBuf::from(env::var("GSVDEC_ROOT").unwrap_or_else(|_| "gsvdec_b200".into()));
    let lib_dir = env::var("GSVDEC_LIB_DIR")
        .map(PathBuf::from)
        .unwrap_or_else(|_| root.join("gpt-sovits-rs_b200").join("_build"));
    if env::var("GSVDEC_SKIP_BUILD").is_err() {
        // nvcc for sm_100a, no multi-backend dispatch, no CPU fallback.
        let status = Command::new(env::var("PYTHON").unwrap_or_else(|_| "python3".into()))
            .arg(root.join("gpt-sovits-rs_b200").join("build.py"))
            .status()
            .expect("running gpt-sovits-rs_b200/build.py (needs nvcc 12.8+ and python3)");
        assert!(status.success(), "libgsvdec build failed");
    }
    println!("cargo:rustc-link-search=native={}", lib_dir.display());
    println!("cargo:rustc-link-lib=dylib=gsvdec");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", lib_dir.display());
    println!("cargo:rerun-if-env-changed=GSVDEC_ROOT");
    println!("cargo:rerun-if-env-changed=GSVDEC_LIB_DIR");
    println!("cargo:rerun-if-env-changed=GSVDEC_SKIP_BUILD");
    println!("cargo:rerun-if-changed={}", root.join("gpt-sovits-rs_b200").join("csrc").display());
    println!("cargo:rerun-if-changed={}", root.join("include").join("gsvdec.h").display());
}
