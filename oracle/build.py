"""Build recipe for the C oracle (test infrastructure): ``python -m oracle.build``.

Compiles ``oracle/lsap.c`` with plain gcc into ``oracle/_build/liboracle_lsap.so``.
``-ffp-contract=off`` and no fast-math keep every float64 operation rounded the
way the C source spells it.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(BUILD_DIR, "liboracle_lsap.so")
SOURCES = [os.path.join(HERE, "lsap.c")]


def build(force: bool = False) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    newest = max(os.path.getmtime(s) for s in SOURCES)
    if not force and os.path.exists(LIB_PATH) and os.path.getmtime(LIB_PATH) >= newest:
        return LIB_PATH
    cmd = ["gcc", "-O2", "-std=c99", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           *SOURCES, "-o", LIB_PATH + ".tmp", "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
