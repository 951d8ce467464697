"""Build libgdn_b200.so in-tree (nvcc, sm_100a) with the Makefile in csrc/."""

from __future__ import annotations

import os
import subprocess

_CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc")


def build(jobs: int = 8) -> str:
    subprocess.run(["make", "-s", "-j", str(jobs), "-C", _CSRC], check=True)
    from . import _lib

    return _lib.LIB_PATH


if __name__ == "__main__":
    print(build())
