"""Build recipe for the CPU oracle (test infrastructure only).

Compiles oracle/oracle.c into oracle/_build/liboracle.so.  The product never loads this
library; tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle.so")


def build(force: bool = False) -> str:
    src = os.path.join(HERE, "oracle.c")
    hdr = os.path.join(HERE, "oracle.h")
    if (not force and os.path.exists(LIB)
            and os.path.getmtime(LIB) >= max(os.path.getmtime(src), os.path.getmtime(hdr))):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
           "-fPIC", "-shared", "-std=c11", "-Wall", "-Wno-unused-function",
           "-Wno-misleading-indentation", "-o", LIB + ".tmp", src, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
