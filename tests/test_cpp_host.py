"""The C++ operator interface (include/onnxb200.hpp), compiled against the
installed header and the in-tree libonnxb200.so: registry, validation and
shape inference on the CPU; compute() of every operator on a GPU
(tests/cpp/test_host_ops.cpp)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "test_host_ops.cpp")


@pytest.fixture(scope="module")
def host_test_bin(ob, tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    if not cxx:
        pytest.skip("no C++ compiler")
    libdir = os.path.dirname(ob.LIB_PATH)
    out = str(tmp_path_factory.mktemp("cpp") / "test_host_ops")
    cmd = [cxx, "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), SRC, "-o", out,
           "-L", libdir, "-lonnxb200", "-Wl,-rpath," + libdir]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    return out


def run(binary, mode):
    r = subprocess.run([binary, mode], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.stdout + r.stderr)[-4000:]
    assert r.stdout.strip().splitlines()[-1].startswith("OK")


def test_cpp_operator_interface_cpu(host_test_bin):
    run(host_test_bin, "cpu")


@pytest.mark.gpu
def test_cpp_operator_interface_gpu(host_test_bin):
    run(host_test_bin, "gpu")
