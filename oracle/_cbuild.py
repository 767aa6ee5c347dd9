"""Builds the oracle's C restatements into ``oracle/_lib/liboracle_c.so``
(test infrastructure only; ``gcc -O2 -ffp-contract=off`` so every fp32 product
and sum is rounded separately, as the restated shader writes them)."""

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(OUT_DIR, "liboracle_c.so")
SOURCES = ["q4_0_gemv.c"]


def build(force: bool = False) -> str:
    srcs = [os.path.join(HERE, s) for s in SOURCES]
    if not force and os.path.exists(LIB) and all(os.path.getmtime(LIB) >= os.path.getmtime(s) for s in srcs):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = ["gcc", "-O2", "-ffp-contract=off", "-fno-fast-math", "-shared", "-fPIC", "-o", LIB, *srcs]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
