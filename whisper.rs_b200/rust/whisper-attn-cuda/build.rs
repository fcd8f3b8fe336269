//! Builds libwattn.so from the CUDA sources with nvcc (sm_100a, static CUDA
//! runtime) and links the crate against it.
//!
//! The sources are the `.cu` files of the library's `csrc` directory:
//! `WATTN_CSRC` if set, else `../../csrc` relative to this crate (its place in
//! the attention repository). Every file of SOURCES is compiled and the build
//! stops if the directory holds a `.cu` file the list does not name, so the
//! library never links with a launcher missing.
use std::{env, fs, path::PathBuf, process::Command};

/// Every CUDA source of the library (csrc/<name>.cu).
const SOURCES: [&str; 7] = [
    "api",
    "attn_f32",
    "attn_tc",
    "decode",
    "decode_noalloc",
    "kv_cache",
    "linear_tc",
];

const ARCH: [&str; 2] = ["-gencode", "arch=compute_100a,code=sm_100a"];

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").expect("CARGO_MANIFEST_DIR"));
    let csrc = env::var_os("WATTN_CSRC")
        .map(PathBuf::from)
        .unwrap_or_else(|| manifest.join("../../csrc"));
    let out = PathBuf::from(env::var("OUT_DIR").expect("OUT_DIR"));
    let nvcc = env::var("NVCC").unwrap_or_else(|_| "nvcc".to_string());

    // The list must name every .cu file of the directory.
    let mut found: Vec<String> = fs::read_dir(&csrc)
        .unwrap_or_else(|e| panic!("cannot read {}: {e}", csrc.display()))
        .filter_map(|e| e.ok())
        .filter_map(|e| {
            let name = e.file_name().into_string().ok()?;
            name.strip_suffix(".cu").map(str::to_string)
        })
        .collect();
    found.sort();
    let mut listed: Vec<String> = SOURCES.iter().map(|s| s.to_string()).collect();
    listed.sort();
    assert_eq!(found, listed, "csrc/*.cu and SOURCES differ");

    let mut objs = Vec::new();
    for name in SOURCES {
        let src = csrc.join(format!("{name}.cu"));
        let obj = out.join(format!("{name}.o"));
        let status = Command::new(&nvcc)
            .args(ARCH)
            .args([
                "-O3",
                "-lineinfo",
                "-std=c++17",
                "-Xcompiler",
                "-fPIC",
                "--expt-relaxed-constexpr",
                "-c",
            ])
            .arg(&src)
            .arg("-o")
            .arg(&obj)
            .status()
            .expect("failed to run nvcc");
        assert!(status.success(), "nvcc failed on {}", src.display());
        println!("cargo:rerun-if-changed={}", src.display());
        objs.push(obj);
    }
    for entry in fs::read_dir(&csrc).expect("csrc").filter_map(|e| e.ok()) {
        let p = entry.path();
        if matches!(p.extension().and_then(|x| x.to_str()), Some("cuh") | Some("h")) {
            println!("cargo:rerun-if-changed={}", p.display());
        }
    }
    let header = csrc.join("../../include/wattn.h");
    println!("cargo:rerun-if-changed={}", header.display());
    println!("cargo:rerun-if-env-changed=WATTN_CSRC");

    let lib = out.join("libwattn.so");
    let status = Command::new(&nvcc)
        .args(ARCH)
        .args(["-shared", "-cudart", "static", "-o"])
        .arg(&lib)
        .args(&objs)
        .status()
        .expect("failed to run nvcc (link)");
    assert!(status.success(), "linking libwattn.so failed");
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=dylib=wattn");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", out.display());
}
