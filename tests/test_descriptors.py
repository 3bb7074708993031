"""tcgen05 descriptor encoders checked against CUTLASS's bit-field definitions (CPU only).

Compiles tests/native/desc_check.cu as host code with the CUTLASS/CuTe headers that ship
inside the flashinfer wheel of this image; skipped where those headers or nvcc are absent.
"""
import glob
import os
import shutil
import subprocess
import sysconfig

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def cutlass_include():
    site = sysconfig.get_paths()["purelib"]
    for pat in ("flashinfer/data/cutlass/include", "tilelang/3rdparty/cutlass/include"):
        for p in glob.glob(os.path.join(site, pat)):
            if os.path.exists(os.path.join(p, "cute", "arch", "mma_sm100_desc.hpp")):
                return p
    return None


def test_descriptors_match_cutlass(tmp_path):
    inc = cutlass_include()
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if inc is None or not os.path.exists(nvcc):
        pytest.skip("CUTLASS headers or nvcc not available")
    exe = str(tmp_path / "desc_check")
    src = os.path.join(ROOT, "tests", "native", "desc_check.cu")
    r = subprocess.run([nvcc, "-std=c++17", "-I", inc, "-I", os.path.join(ROOT, "kandinsky.cpp_b200", "csrc"),
                        "-o", exe, src], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.strip() == "OK", out.stdout + out.stderr
