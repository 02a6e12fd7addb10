// Compiles ../../csrc/*.cu for sm_100a into a static library: each source
// with relocatable device code, one device-link object over all of them,
// then `ar` -- the same recipe as rust-cev_b200/build.py --static.  The
// final link needs the CUDA runtime and driver and libstdc++.
use std::path::{Path, PathBuf};
use std::process::Command;

fn run(cmd: &mut Command, what: &str) {
    let st = cmd.status().unwrap_or_else(|e| panic!("{what}: {e}"));
    assert!(st.success(), "{what} failed");
}

fn main() {
    let here = PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").unwrap());
    let csrc = here.join("../../csrc");
    let include = here.join("../../../include");
    let out = PathBuf::from(std::env::var("OUT_DIR").unwrap());
    let nvcc = std::env::var("NVCC").unwrap_or_else(|_| "nvcc".into());
    let arch = ["-gencode", "arch=compute_100a,code=sm_100a"];
    let mut objs: Vec<PathBuf> = Vec::new();
    let mut srcs: Vec<PathBuf> = std::fs::read_dir(&csrc)
        .unwrap()
        .map(|e| e.unwrap().path())
        .filter(|p| p.extension().is_some_and(|e| e == "cu"))
        .collect();
    srcs.sort();
    for src in &srcs {
        let obj = out.join(Path::new(src.file_stem().unwrap()).with_extension("o"));
        run(
            Command::new(&nvcc)
                .args(arch)
                .args(["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"])
                .args(["-diag-suppress", "20044", "-I"])
                .arg(&include)
                .arg("-c")
                .arg(src)
                .arg("-o")
                .arg(&obj),
            "nvcc -c",
        );
        objs.push(obj);
        println!("cargo:rerun-if-changed={}", src.display());
    }
    let dlink = out.join("cevk_dlink.o");
    run(Command::new(&nvcc).args(arch).args(["-dlink", "-Xcompiler", "-fPIC"]).args(&objs).arg("-o").arg(&dlink), "nvcc -dlink");
    let lib = out.join("libcevk.a");
    let _ = std::fs::remove_file(&lib);
    run(Command::new("ar").arg("rcs").arg(&lib).args(&objs).arg(&dlink), "ar");
    println!("cargo:rerun-if-changed={}", csrc.join("common.cuh").display());
    println!("cargo:rerun-if-changed={}", include.join("cevk.h").display());
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=static=cevk");
    let cuda = std::env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into());
    println!("cargo:rustc-link-search=native={cuda}/lib64");
    println!("cargo:rustc-link-lib=dylib=cudart");
    println!("cargo:rustc-link-lib=dylib=cuda");
    println!("cargo:rustc-link-lib=dylib=stdc++");
}
