// build.rs -- with the `build-cuda` feature, compile libswamp_gpu.so for
// sm_100a from the CUDA sources (one translation unit, csrc/swamp_gpu.cu)
// with nvcc into OUT_DIR, and tell the crate where it is. Without the
// feature (or without nvcc) nothing is built and the library is looked up
// at run time (see src/lib.rs). The reference crate's build.rs ran `make`
// on its own kernels (swamp-gpu/build.rs:8-29); this one replaces it.
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    println!("cargo:rerun-if-env-changed=SWAMP_GPU_SRC");
    println!("cargo:rerun-if-env-changed=NVCC");
    if env::var_os("CARGO_FEATURE_BUILD_CUDA").is_none() {
        return;
    }
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    // the CUDA sources: SWAMP_GPU_SRC, else the repository's own csrc next to
    // this crate (rust/swamp-gpu -> ../../llamanyon.rs_b200/csrc)
    let src = env::var_os("SWAMP_GPU_SRC")
        .map(PathBuf::from)
        .unwrap_or_else(|| manifest.join("../../llamanyon.rs_b200/csrc"));
    let unit = src.join("swamp_gpu.cu");
    println!("cargo:rerun-if-changed={}", src.display());
    let nvcc = env::var("NVCC").unwrap_or_else(|_| "nvcc".to_string());
    let out = PathBuf::from(env::var("OUT_DIR").unwrap()).join("libswamp_gpu.so");
    let status = Command::new(&nvcc)
        .args([
            "-gencode", "arch=compute_100a,code=sm_100a",
            "-O3", "-lineinfo", "-std=c++17",
            "-Xcompiler", "-fPIC,-O2,-fvisibility=hidden",
            "-shared", "-cudart", "shared",
            "-diag-suppress", "177",
            "-o",
        ])
        .arg(&out)
        .arg(&unit)
        .arg("-ldl")
        .status();
    match status {
        Ok(s) if s.success() => {
            println!("cargo:rustc-env=SWAMP_GPU_LIB={}", out.display());
        }
        Ok(s) => panic!("nvcc failed ({s}) building {}", unit.display()),
        Err(e) => println!("cargo:warning=nvcc not runnable ({e}); libswamp_gpu.so must be found at run time"),
    }
}
