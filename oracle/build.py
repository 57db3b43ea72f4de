"""Compile the C restatement of the oracle (titan_oracle.c) with gcc.

Output: oracle/_build/libtitan_oracle.so.  -O2 without -ffast-math, so fp32
division and rintf keep their IEEE round-to-nearest-even meaning.  The
reference itself is Python + Triton with no C/C++ sources, so there is no
oracle/_ref build.
"""
import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "titan_oracle.c"
OUT = HERE / "_build" / "libtitan_oracle.so"


def build(force=False):
    if not force and OUT.exists() and OUT.stat().st_mtime >= SRC.stat().st_mtime:
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    subprocess.run(["gcc", "-O2", "-std=c11", "-fno-fast-math", "-ffp-contract=off", "-fPIC", "-shared",
                    "-o", str(tmp), str(SRC), "-lm"], check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
