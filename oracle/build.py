"""Build the CPU oracle (test infrastructure only) into oracle/_build/liboracle.so.

gcc -O2 -ffp-contract=off: every f32 multiply and add rounds on its own, as
in the Rust code being restated (rustc never contracts to FMA). -fopenmp
gives the rayon-style parallel loops; each output is computed by one thread,
so results do not depend on the thread count.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle.so")


def build(force: bool = False) -> str:
    src = os.path.join(HERE, "oracle.c")
    hdr = os.path.join(HERE, "oracle.h")
    os.makedirs(OUT_DIR, exist_ok=True)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(src), os.path.getmtime(hdr)):
        return LIB
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-fopenmp",
           src, "-o", LIB, "-lm"]
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv)
