"""The error bound of CUDA's expf that the exact-sum classification relies on.

The kernels classify each element by CUDA's expf(d) and replace it by libm's value
wherever the two could round differently, judging "could" with a relative error bound
of 2^-21 (lrs_kernels.cu: classify_elem, classify_pair1; warp_serial_add).  This test
measures CUDA's expf against the double-precision exp over every float d in [-104, 0)
with a normal result, on this GPU and toolchain, and checks the bound with room to spare.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

from lrs import build as B

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_cuda_expf_relative_error_below_the_classification_bound(tmp_path):
    lib = tmp_path / "expf_bound.so"
    subprocess.run([B.nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-shared", "-Xcompiler", "-fPIC",
                    os.path.join(HERE, "csrc", "expf_bound.cu"), "-o", str(lib)], check=True)
    out = np.zeros(104, np.uint32)
    rc = ctypes.CDLL(str(lib)).lrs_test_expf_error(out.ctypes.data_as(ctypes.c_void_p))
    assert rc == 0
    err = out.view(np.float32)
    worst = float(err.max())
    assert worst > 0.0                       # the probe ran
    assert worst < 2.0 ** -21 / 2            # the classification's 2^-21, with a factor 2 to spare


def test_branch_free_double_exp_against_cuda_double_exp(tmp_path):
    # lrs::exp_neg (Cody-Waite reduction, Taylor degree 12) stands in for the double exp of the
    # correctly rounded float exp: within 1e-14 relative of CUDA's double exp over every float
    # d in [-104, 0), and never rounding to another float where the midpoint test trusts it.
    lib = tmp_path / "exp_neg_bound.so"
    subprocess.run([B.nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-shared",
                    "-Xcompiler", "-fPIC", os.path.join(HERE, "csrc", "exp_neg_bound.cu"), "-o", str(lib)],
                   check=True)
    out = np.zeros(2, np.uint32)
    rc = ctypes.CDLL(str(lib)).lrs_test_exp_neg(out.ctypes.data_as(ctypes.c_void_p))
    assert rc == 0
    worst = float(out[:1].view(np.float32)[0])
    assert 0.0 < worst < 1e-14
    assert out[1] == 0
