"""Build recipe for the native library (nvcc, sm_100a), in-tree.

``build()`` runs the Makefile in tinygnn_b200/csrc, which compiles every
kernel with ``-gencode arch=compute_100a,code=sm_100a -lineinfo`` into
tinygnn_b200/lib/libtinygnn_b200.so, then the pybind11 module
tinygnn_b200/tinygnn/_core (TinyGNN's Python API over the C++ API in that
library).  No GPU is needed to build.

This file imports nothing from the package, so it can be loaded by path
(``__graft_entry__.build()``) before the library exists; the package's
loader calls :func:`ensure_built` when the library is missing.  Builds are
serialised across processes with a lock file (several ranks started by
torchrun may import the package at once).
"""
from __future__ import annotations

import contextlib
import fcntl
import os
import shutil
import subprocess
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libtinygnn_b200.so")
PYMOD_DIR = os.path.join(HERE, "tinygnn")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def pymodule_path() -> str:
    return os.path.join(PYMOD_DIR, "_core" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def _python_flags() -> list[str]:
    import pybind11
    incs = {sysconfig.get_paths()["include"], sysconfig.get_paths()["platinclude"], pybind11.get_include()}
    return [f"PY_INCLUDES={' '.join('-I' + i for i in sorted(incs))}",
            f"PY_EXT={sysconfig.get_config_var('EXT_SUFFIX')}"]


@contextlib.contextmanager
def _lock():
    os.makedirs(LIB_DIR, exist_ok=True)
    with open(os.path.join(LIB_DIR, ".build.lock"), "w") as f:
        fcntl.flock(f, fcntl.LOCK_EX)
        try:
            yield
        finally:
            fcntl.flock(f, fcntl.LOCK_UN)


def _make(args: list[str], quiet: bool) -> None:
    r = subprocess.run(["make", "-C", CSRC, *args], stdout=subprocess.PIPE if quiet else None,
                       stderr=subprocess.STDOUT if quiet else None, text=True)
    if r.returncode != 0:
        tail = (r.stdout or "")[-4000:]
        raise RuntimeError(f"tinygnn_b200: building the native library failed (make {' '.join(args)}):\n{tail}")


def build(jobs: int = 0, quiet: bool = True) -> str:
    """Compile (or bring up to date) the library and the Python module."""
    jobs = jobs or min(32, os.cpu_count() or 8)
    with _lock():
        _make([f"-j{jobs}"], quiet)
        _make(["pymodule", *_python_flags()], quiet)
    return LIB_PATH


def ensure_built(pymodule: bool = False) -> str:
    """Build the library (and, if asked, the Python module) when it is
    missing.  Raises ImportError when it is missing and nvcc is not there
    to build it: the package has no CPU path."""
    want = [LIB_PATH] + ([pymodule_path()] if pymodule else [])
    if all(os.path.exists(p) for p in want):
        return LIB_PATH
    if not (os.path.exists(NVCC) or shutil.which("nvcc")):
        raise ImportError(f"tinygnn_b200: {LIB_PATH} is missing and nvcc is not available to build it "
                          "(there is no CPU fallback)")
    with _lock():
        if all(os.path.exists(p) for p in want):  # another process built it meanwhile
            return LIB_PATH
    try:
        build()
    except RuntimeError as e:
        raise ImportError(str(e)) from e
    return LIB_PATH


if __name__ == "__main__":
    print(build(quiet=False))
