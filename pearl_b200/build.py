"""Build recipe for the pearl_b200 CUDA library (in-tree, sm_100a only).

    python -m pearl_b200.build          # or: python pearl_b200/build.py

Produces pearl_b200/_lib/libpearl_b200.so with nvcc (static cudart, no torch
dependency) and writes the ptxas register/spill report next to it.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_DIR = os.path.join(HERE, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libpearl_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the pearl_b200 CUDA library cannot be built")
    return path


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def needs_rebuild() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = sources() + glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + [
        os.path.join(ROOT, "include", "pearl_b200.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_rebuild():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    cmd = [nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-cudart", "static",
           "-Xptxas", "-v", "-I", os.path.join(ROOT, "include"),
           "-o", LIB_PATH + ".tmp", *sources()]
    res = subprocess.run(cmd, capture_output=True, text=True)
    with open(os.path.join(LIB_DIR, "ptxas_report.txt"), "w") as f:
        f.write(" ".join(cmd) + "\n\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libpearl_b200.so")
    if verbose:
        sys.stdout.write(res.stderr)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
