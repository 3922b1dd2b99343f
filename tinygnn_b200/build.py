"""Build recipe for the native library (nvcc, sm_100a), in-tree.

``build()`` runs the Makefile in tinygnn_b200/csrc, which compiles every
kernel with ``-gencode arch=compute_100a,code=sm_100a -lineinfo`` into
tinygnn_b200/lib/libtinygnn_b200.so, then the pybind11 module
tinygnn_b200/tinygnn/_core (TinyGNN's Python API over the C++ API in that
library).  No GPU is needed to build.
"""
from __future__ import annotations

import os
import subprocess
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))


def _python_flags() -> list[str]:
    import pybind11
    incs = {sysconfig.get_paths()["include"], sysconfig.get_paths()["platinclude"], pybind11.get_include()}
    return [f"PY_INCLUDES={' '.join('-I' + i for i in sorted(incs))}",
            f"PY_EXT={sysconfig.get_config_var('EXT_SUFFIX')}"]


def build(jobs: int = 8, quiet: bool = True) -> str:
    out = subprocess.DEVNULL if quiet else None
    csrc = os.path.join(HERE, "csrc")
    subprocess.run(["make", "-C", csrc, f"-j{jobs}"], check=True, stdout=out)
    subprocess.run(["make", "-C", csrc, "pymodule", *_python_flags()], check=True, stdout=out)
    return os.path.join(HERE, "lib", "libtinygnn_b200.so")


if __name__ == "__main__":
    print(build(quiet=False))
