"""exp2_poly (part of the softmax exponentials on the FMA pipe) against exp2 in double, on the GPU, and
its packed f32x2 form exp2_poly2 against it bit for bit.

Bound: 2^-13 relative error over the softmax's argument range (the Remez fit gives 7.5e-5 =
2^-13.7 before float rounding), exact zeros at or below -126 and for -inf.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def test_exp2_poly_error_bound(tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = str(tmp_path / "exp2_check")
    r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                        "-I", os.path.join(ROOT, "kandinsky.cpp_b200", "csrc"),
                        os.path.join(ROOT, "tests", "native", "exp2_check.cu"), "-o", exe],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    fields = out.stdout.split()
    max_rel, zero_ok, pair_equal = float(fields[1]), int(fields[3]), int(fields[5])
    assert zero_ok == 1
    assert pair_equal == 1, "exp2_poly2 differs from exp2_poly"
    assert max_rel <= 2.0 ** -13, max_rel
