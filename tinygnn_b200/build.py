"""Build recipe for the native library (nvcc, sm_100a), in-tree.

``build()`` runs the Makefile in tinygnn_b200/csrc, which compiles every
kernel with ``-gencode arch=compute_100a,code=sm_100a -lineinfo`` into
tinygnn_b200/lib/libtinygnn_b200.so.  No GPU is needed to build.
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 8, quiet: bool = True) -> str:
    subprocess.run(["make", "-C", os.path.join(HERE, "csrc"), f"-j{jobs}"], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)
    return os.path.join(HERE, "lib", "libtinygnn_b200.so")


if __name__ == "__main__":
    print(build(quiet=False))
