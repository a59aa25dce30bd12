//! Compiles libraya_attn for sm_100a with nvcc and links it.
//!
//! RAYA_B200_ROOT must point at a checkout of the raya_b200 repository (the
//! directory holding `include/raya_attn.h` and `raya_b200/csrc/`); NVCC may
//! name the compiler (default `nvcc` on PATH).  The command is the one
//! `python raya_b200/build.py` runs.
use std::{env, path::PathBuf, process::Command};

fn main() {
    let root = PathBuf::from(
        env::var("RAYA_B200_ROOT").expect("set RAYA_B200_ROOT to the raya_b200 checkout (include/, raya_b200/csrc/)"),
    );
    let out = PathBuf::from(env::var("OUT_DIR").expect("OUT_DIR is set by cargo"));
    let nvcc = env::var("NVCC").unwrap_or_else(|_| "nvcc".to_string());
    let source = root.join("raya_b200").join("csrc").join("raya_attn.cu");
    let status = Command::new(&nvcc)
        .args([
            "-gencode",
            "arch=compute_100a,code=sm_100a",
            "-O3",
            "-lineinfo",
            "-std=c++17",
            "--expt-relaxed-constexpr",
            "-Xcompiler",
            "-fPIC",
            "-shared",
            "-cudart",
            "static",
        ])
        .arg("-I")
        .arg(root.join("include"))
        .arg("-o")
        .arg(out.join("libraya_attn.so"))
        .arg(&source)
        .status()
        .unwrap_or_else(|e| panic!("could not run {nvcc}: {e}"));
    assert!(status.success(), "nvcc failed on {}", source.display());
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=dylib=raya_attn");
    // Binaries and tests find the library next to the build output.
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", out.display());
    println!("cargo:rerun-if-env-changed=RAYA_B200_ROOT");
    println!("cargo:rerun-if-env-changed=NVCC");
    println!("cargo:rerun-if-changed={}", root.join("raya_b200").join("csrc").display());
    println!("cargo:rerun-if-changed={}", root.join("include").join("raya_attn.h").display());
}
