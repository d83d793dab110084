"""Build recipe of the in-tree CUDA library (sm_100a only).

``build()`` runs the Makefile in ``csrc/`` (nvcc -gencode arch=compute_100a,code=sm_100a) and
writes ``densecore_b200/libdensecore_sdpa.so``; object files go to ``_build/`` at the repo root.
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs: int = 4, verbose: bool = False) -> str:
    cmd = ["make", "-C", os.path.join(HERE, "csrc"), f"-j{jobs}"]
    if not verbose:
        cmd.insert(1, "-s")
    subprocess.run(cmd, check=True)
    return os.path.join(HERE, "libdensecore_sdpa.so")


if __name__ == "__main__":
    print(build(verbose=True))
