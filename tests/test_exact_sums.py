"""CPU test of the exact sequential-f32 emulation the kernels use (tests/csrc/acc_emul.cpp):
the kernel's grid arithmetic (llama.rs_b200/csrc/lrs_grid.h) replayed serially must give
bit-identical results to plain sequential f32 sums, top-p style stops and draws."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "llama.rs_b200", "csrc")


def test_exact_sum_emulation(tmp_path):
    exe = tmp_path / "acc_emul"
    subprocess.run(["g++", "-O2", "-std=c++17", "-fno-fast-math", "-ffp-contract=off", f"-I{CSRC}",
                    os.path.join(HERE, "csrc", "acc_emul.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
