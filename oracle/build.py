"""Build recipe for the CPU oracle shared library (test infrastructure only).

    python oracle/build.py            # -> oracle/_build/libnq_oracle.so

gcc, -O2, no -ffast-math, -ffp-contract=off: every fp32 operation in
nq_oracle.c is a single IEEE-754 operation, which is what the bit-exact
quantize / dequantize comparisons need.  OpenMP parallelises the row loops
(the qmm CPU baseline uses every host thread).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "nq_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libnq_oracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB + ".tmp%d" % os.getpid()
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-fno-fast-math", "-std=c11", "-Wall", "-o", tmp, SRC, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
