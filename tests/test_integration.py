"""integration/ (the kandinsky.cpp side of the drop-in: ops_kd::attention, the fused DiT node, the
batch-2 CFG pairing) compiled against the declarations-only ggml stub and run with a fake ggml
graph builder and a fake libkd_attn -- no ggml, no GPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_integration_shim_builds_and_maps_like_the_reference(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = str(tmp_path / "integration_test")
    cmd = [gxx, "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "integration", "stub"), "-I", os.path.join(ROOT, "integration"),
           "-I", os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "native", "integration_test.cpp"),
           "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    out = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0 and out.stdout.strip().endswith("ALL OK"), out.stdout + out.stderr
