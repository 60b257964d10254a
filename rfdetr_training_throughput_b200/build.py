"""Build recipe for ``librfm.so`` (sm_100a): ``python -m rfdetr_training_throughput_b200.build``.

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` into one shared library
next to this file (in-tree, so it travels with the repository snapshot).  The
CUDA runtime is linked statically: the library carries its own runtime and
binds to the process's primary context, which it shares with torch.
"""

from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "librfm.so")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr"]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def _inputs() -> list[str]:
    return sources() + glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    newest = max(os.path.getmtime(p) for p in _inputs())
    return os.path.getmtime(LIB_PATH) >= newest


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and up_to_date():
        return LIB_PATH
    out_tmp = LIB_PATH + ".tmp"
    cmd = [NVCC, *ARCH_FLAGS, *FLAGS, *(extra or []), "-I", INCLUDE, "-shared", *sources(), "-o", out_tmp]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(out_tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    extra = ["-Xptxas", "-v"] if "--ptxas" in sys.argv else None
    print(build(force=True, verbose=True, extra=extra))
