"""The C++ host mirror (include/glacier_b200.hpp) compiles against the C ABI and
its host-only paths work; the GPU variant runs one expert through it."""
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(REPO, "tests", "cpp", "host_api_check.cpp")
LIBDIR = os.path.join(REPO, "glacier", "inference", "distributed_b200")


def _build(tmp_path):
    exe = str(tmp_path / "host_api_check")
    subprocess.check_call(["g++", "-std=c++17", "-O1", "-I", os.path.join(REPO, "include"), SRC, "-o", exe,
                           "-L", LIBDIR, "-lglacier_b200", f"-Wl,-rpath,{LIBDIR}"])
    return exe


def test_cpp_host_api_cpu(glc, tmp_path):
    out = subprocess.run([_build(tmp_path), "cpu"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr


@pytest.mark.gpu
def test_cpp_host_api_gpu(cuda, tmp_path):
    out = subprocess.run([_build(tmp_path), "gpu"], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
