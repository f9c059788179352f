"""Builds tests/cpp/test_cpp_api.cpp against libllmx_attn.so and runs it on
the GPU: the reference's C++ tensor and attention tests, restated without
gtest (see the C++ file)."""
import os
import subprocess

import pytest


from gpu_helpers import needs_cuda

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_test_binary():
    from llmx_b200 import build as b

    lib = b.build()
    out = os.path.join(ROOT, "llmx_b200", "_build", "test_cpp_api")
    src = os.path.join(ROOT, "tests", "cpp", "test_cpp_api.cpp")
    cmd = [b.nvcc(), "-std=c++17", "-O2", "-x", "cu", "-I" + os.path.join(ROOT, "include"), src, "-o", out,
           "-L" + os.path.dirname(lib), "-lllmx_attn", "-Xlinker", "-rpath=" + os.path.dirname(lib)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return out


def test_cpp_api_builds():
    assert os.path.exists(build_test_binary())


@pytest.mark.gpu
@needs_cuda
def test_cpp_api_runs():
    exe = build_test_binary()
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all C++ API checks passed" in r.stdout
