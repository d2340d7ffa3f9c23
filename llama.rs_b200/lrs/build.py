"""Build step of the sampler library (no GPU needed: nvcc cross-compiles sm_100a).

Produces, inside the package directory llama.rs_b200/:
  libllamars_sampler.so      the C ABI of include/llamars_sampler.h (CUDA kernels + host code)
  data/expf_glibc.bin        this machine's libm expf exceptions (see csrc/gen_expf_table.c)
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPO = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB = os.path.join(PKG_DIR, "libllamars_sampler.so")
TABLE = os.path.join(PKG_DIR, "data", "expf_glibc.bin")
GEN = os.path.join(PKG_DIR, "data", "gen_expf_table")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC,-O2",
    "-Xptxas", "-warn-spills",
]
SOURCES = ["lrs_kernels.cu", "lrs_api.cu", "lrs_noalloc.cu", "lrs_generate.cu"]
HEADERS = ["lrs_device.cuh", "lrs_grid.h", "lrs_kernels_decl.cuh", "lrs_stages.cuh"]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def build_table(force: bool = False) -> str:
    src = os.path.join(CSRC, "gen_expf_table.c")
    os.makedirs(os.path.dirname(TABLE), exist_ok=True)
    if force or not _newer(TABLE, [src]):
        subprocess.run(["gcc", "-O2", "-fno-fast-math", "-ffp-contract=off", src, "-o", GEN, "-lm", "-pthread"],
                       check=True)
        subprocess.run([GEN, TABLE], check=True)
    return TABLE


def build_lib(force: bool = False, verbose: bool = False) -> str:
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [os.path.join(REPO, "include", "llamars_sampler.h")]
    if force or not _newer(LIB, deps):
        cmd = [nvcc(), *NVCC_FLAGS, "-shared", *[os.path.join(CSRC, s) for s in SOURCES], "-o", LIB, "-ldl"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


def build(force: bool = False, verbose: bool = False) -> str:
    build_table(force)
    return build_lib(force, verbose)


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
