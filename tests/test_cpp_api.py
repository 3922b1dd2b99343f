"""The C++ tinygnn:: API (include/tinygnn/*.hpp, compiled into
libtinygnn_b200.so): it builds against the headers here, and on a GPU the
test program (tests/cpp/test_cpp_api.cpp) passes TinyGNN's known answers."""
import os
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "tinygnn_b200", "lib")
SRC = os.path.join(ROOT, "tests", "cpp", "test_cpp_api.cpp")


def _build(out):
    cmd = ["/usr/bin/g++", "-std=c++17", "-O1", SRC, "-I", os.path.join(ROOT, "include"),
           "-I", "/usr/local/cuda/include", "-L", LIBDIR, "-ltinygnn_b200",
           f"-Wl,-rpath,{LIBDIR}", "-Wl,-rpath,/usr/local/cuda/lib64", "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]


def test_cpp_api_builds_against_the_headers():
    with tempfile.TemporaryDirectory() as d:
        _build(os.path.join(d, "t"))


@pytest.mark.gpu
def test_cpp_api_known_answers_on_device():
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "t")
        _build(exe)
        r = subprocess.run([exe, d], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
        assert "0 failed" in r.stdout
