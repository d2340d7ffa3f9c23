//! Builds (or links) libllamars_sampler.so, the CUDA library behind the FFI in src/ffi.rs.
//!
//! * `LLAMARS_SAMPLER_LIB_DIR=<dir>`: link the library already built there (for example by
//!   `python llama.rs_b200/lrs/build.py`, which writes llama.rs_b200/libllamars_sampler.so and
//!   llama.rs_b200/data/expf_glibc.bin).
//! * otherwise: compile ../llama.rs_b200/csrc/*.cu with nvcc for sm_100a into OUT_DIR, and
//!   generate OUT_DIR/data/expf_glibc.bin (this machine's libm expf exceptions, which the
//!   library loads from `data/` next to itself, or from LRS_EXPF_TABLE).
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn run(cmd: &mut Command) {
    let status = cmd.status().unwrap_or_else(|e| panic!("failed to run {cmd:?}: {e}"));
    assert!(status.success(), "{cmd:?} failed with {status}");
}

fn main() {
    println!("cargo:rerun-if-env-changed=LLAMARS_SAMPLER_LIB_DIR");
    println!("cargo:rerun-if-env-changed=NVCC");
    if let Ok(dir) = env::var("LLAMARS_SAMPLER_LIB_DIR") {
        println!("cargo:rustc-link-search=native={dir}");
        println!("cargo:rustc-link-lib=dylib=llamars_sampler");
        println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
        return;
    }
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let csrc = manifest.join("../llama.rs_b200/csrc");
    let include = manifest.join("../include");
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());
    let nvcc = env::var("NVCC").unwrap_or_else(|_| "/usr/local/cuda/bin/nvcc".into());
    let sources = ["lrs_kernels.cu", "lrs_api.cu", "lrs_noalloc.cu"];
    for f in sources
        .iter()
        .chain(["lrs_device.cuh", "lrs_grid.h", "lrs_kernels_decl.cuh", "lrs_stages.cuh", "gen_expf_table.c"].iter())
    {
        println!("cargo:rerun-if-changed={}", csrc.join(f).display());
    }
    println!("cargo:rerun-if-changed={}", include.join("llamars_sampler.h").display());
    let mut cmd = Command::new(&nvcc);
    cmd.args(["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo"])
        .args(["-Xcompiler", "-fPIC,-O2", "-shared"]);
    for s in sources {
        cmd.arg(csrc.join(s));
    }
    cmd.arg("-o").arg(out.join("libllamars_sampler.so")).arg("-ldl");
    run(&mut cmd);
    // the libm expf exception table, generated from this machine's libm
    let data = out.join("data");
    std::fs::create_dir_all(&data).unwrap();
    let gen = out.join("gen_expf_table");
    run(Command::new("gcc")
        .args(["-O2", "-fno-fast-math", "-ffp-contract=off"])
        .arg(csrc.join("gen_expf_table.c"))
        .arg("-o")
        .arg(&gen)
        .args(["-lm", "-pthread"]));
    run(Command::new(&gen).arg(data.join("expf_glibc.bin")));
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=dylib=llamars_sampler");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", out.display());
}
