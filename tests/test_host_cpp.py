"""The C++ host layer (kandinsky.cpp_b200/host/kd_ops.hpp: ops::attention, dit_self_attention,
dit_cross_attention over the C ABI) built with g++ and run: host-side checks on any machine,
the GPU path against the oracle's C restatement on a B200."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build_test(kd, tmp_path):
    """g++ -> tests/native/host_ops_test linked against libkd_attn.so, the oracle and cudart."""
    from oracle.build_oracle import build_oracle
    oracle_lib = build_oracle()
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    lib_dir = os.path.dirname(kd.LIB_PATH)
    exe = str(tmp_path / "host_ops_test")
    cmd = [gxx, "-std=c++17", "-O2", "-Wall", "-Wextra",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "kandinsky.cpp_b200", "host"),
           "-I", os.path.join(ROOT, "oracle"), "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "native", "host_ops_test.cpp"), "-o", exe,
           kd.LIB_PATH, oracle_lib, "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{os.path.dirname(oracle_lib)}",
           f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    return exe


def test_host_layer_builds_and_host_checks_pass(kd, tmp_path):
    exe = build_test(kd, tmp_path)
    out = subprocess.run([exe, "--cpu"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip().endswith("OK"), out.stdout + out.stderr


@pytest.mark.gpu
def test_host_layer_matches_oracle_on_gpu(kd, tmp_path):
    exe = build_test(kd, tmp_path)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    print(out.stdout)
    assert out.returncode == 0 and out.stdout.strip().endswith("OK"), out.stdout + out.stderr
