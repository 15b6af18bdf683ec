"""Build the in-tree CUDA library for B200 (sm_100a).

``python -m stealcode_b200.build`` runs nvcc through ``stealcode_b200/csrc/Makefile``
(``-gencode arch=compute_100a,code=sm_100a -lineinfo``, no fast-math) and
leaves ``stealcode_b200/libstealcode_cuda.so`` next to this file, where the
ctypes binding loads it.  nvcc cross-compiles, so no GPU is needed to build.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")


def build(jobs: int = 8) -> str:
    subprocess.run(["make", "-s", "-j", str(jobs), "-C", CSRC], check=True)
    return os.path.join(HERE, "libstealcode_cuda.so")


if __name__ == "__main__":
    print(build(int(sys.argv[1]) if len(sys.argv) > 1 else 8))
