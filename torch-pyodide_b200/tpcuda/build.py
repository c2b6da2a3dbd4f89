"""Build libtpcuda.so in-tree with nvcc for sm_100a (csrc/Makefile)."""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "csrc")


def build(jobs: int | None = None, verbose: bool = False) -> str:
    """Compile every CUDA source under csrc/ and link tpcuda/libtpcuda.so."""
    jobs = jobs or max(1, min(16, os.cpu_count() or 1))
    cmd = ["make", "-C", CSRC, f"-j{jobs}"]
    if not verbose:
        cmd.insert(1, "-s")
    subprocess.run(cmd, check=True)
    return os.path.join(HERE, "libtpcuda.so")
