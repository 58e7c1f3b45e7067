"""The reference's C++ API (namespace aaedn, project-aaedn_b200/host/include)
compiled against the library as a reference-side caller would: the
startup-failure checks of the reference's own tests/test_startup_failure.cpp
on CPU, and every API function on a GPU (tests/cpp/test_api_gpu.cpp)."""
import os
import subprocess

import pytest

import aaedn_b200 as ab

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _build(src, out):
    lib = ab.LIB_PATH
    cmd = ["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(ROOT, "project-aaedn_b200", "host", "include"),
           "-I", os.path.join(ROOT, "tests", "cpp"), os.path.join(ROOT, "tests", "cpp", src), "-o", str(out),
           lib, "-Wl,-rpath," + os.path.dirname(lib)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def _run(exe, tmp_path):
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "PASSED" in r.stdout, r.stdout + r.stderr


def test_startup_failure_cpu(tmp_path):
    exe = tmp_path / "test_startup_failure"
    _build("test_startup_failure.cpp", exe)
    _run(exe, tmp_path)


@pytest.mark.gpu
def test_cpp_api_on_gpu(tmp_path):
    exe = tmp_path / "test_api_gpu"
    _build("test_api_gpu.cpp", exe)
    _run(exe, tmp_path)
