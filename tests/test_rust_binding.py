"""The Rust crate's view of the C ABI (rust/src/ffi.rs), checked on the CPU: the same
function names as tests/csrc/rust_abi.c (which mirrors the Rust signatures and is compiled
against include/llamars_sampler.h with -Werror), each declared in the header and exported by
the built library.  The crate itself is not compiled here: the image has no Rust toolchain."""
import os
import re
import subprocess

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def rust_functions():
    src = open(os.path.join(REPO, "rust", "src", "ffi.rs")).read()
    block = src[src.index('extern "C" {'):]
    return set(re.findall(r"\bpub fn (lrs_[a-z0-9_]+)\s*\(", block))


def c_mirror_functions():
    src = open(os.path.join(REPO, "tests", "csrc", "rust_abi.c")).read()
    return set(re.findall(r"typedef [^;]*?\(\*rs_(lrs_[a-z0-9_]+)\)", src))


def test_rust_ffi_and_c_mirror_name_the_same_functions():
    rs = rust_functions()
    assert len(rs) >= 16
    assert rs == c_mirror_functions()


def test_rust_abi_mirror_compiles_against_the_header_and_binds_the_library(built_lib, tmp_path):
    exe = str(tmp_path / "rust_abi")
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-Werror=incompatible-pointer-types",
                    os.path.join(REPO, "tests", "csrc", "rust_abi.c"), "-o", exe, "-ldl"], check=True)
    out = subprocess.run([exe, built_lib], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert "rust ABI ok" in out.stdout
