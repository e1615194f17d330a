"""Builds libshahd_b200.so in-tree with nvcc for sm_100a (cross-compiles without a GPU).

    python -m shahd-llm-stack_b200.build        (or importlib: build.build())
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
SO_PATH = os.path.join(HERE, "libshahd_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _sources() -> list[str]:
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files.append(os.path.join(INCLUDE, "shahd_b200.h"))
    return files


def up_to_date() -> bool:
    if not os.path.exists(SO_PATH):
        return False
    t = os.path.getmtime(SO_PATH)
    return all(os.path.getmtime(f) <= t for f in _sources())


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    """Compile the library unless it is newer than every source; returns the .so path."""
    if not force and up_to_date():
        return SO_PATH
    nvcc = os.environ.get("NVCC", "nvcc")
    tmp = SO_PATH + ".tmp"
    cmd = [nvcc, *NVCC_FLAGS, *(extra or []), "-o", tmp, os.path.join(CSRC, "shahd_b200.cu")]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, SO_PATH)
    return SO_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
