"""Build the in-tree native libraries (nvcc for sm_100a, g++ for the host)."""

from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def library_path(name: str = "libvolta_cuda_backend.so") -> str:
    return os.path.join(HERE, name)


def build_all(jobs: int = 8) -> None:
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", os.path.join(HERE, "csrc")], check=True)
    subprocess.run(["make", "-s", "-C", os.path.join(HERE, "host")], check=True)
