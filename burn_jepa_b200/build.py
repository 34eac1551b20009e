"""Builds libbjf.so in-tree for sm_100a (nvcc via burn_jepa_b200/csrc/Makefile)."""
from __future__ import annotations

import os
import subprocess

_PKG = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 8) -> str:
    """Compiles every CUDA/C++ source of the library (-gencode arch=compute_100a,code=sm_100a)."""
    subprocess.run(["make", "-s", "-C", os.path.join(_PKG, "csrc"), f"-j{jobs}"], check=True)
    return os.path.join(_PKG, "libbjf.so")


if __name__ == "__main__":
    print(build())
