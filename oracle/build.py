"""Build recipe for the CPU oracle (test infrastructure only).

Compiles oracle/hyq_oracle.c into oracle/libhyq_oracle.so with gcc.  The
flags keep Rust's floating-point semantics: -ffp-contract=off (no implicit
FMA; the reference's FMA intrinsics are written as fmaf) and no fast-math.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "hyq_oracle.c")
OUT = os.path.join(HERE, "libhyq_oracle.so")

FLAGS = ["-O2", "-mavx2", "-mfma", "-ffp-contract=off", "-fno-fast-math", "-fopenmp",
         "-fPIC", "-shared", "-std=c11", "-Wall", "-Wextra", "-Wno-unused-parameter"]


def build(force: bool = False) -> str:
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    tmp = OUT + ".tmp"
    subprocess.check_call(["gcc", *FLAGS, SRC, "-o", tmp, "-lm"])
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
