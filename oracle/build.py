"""Build the CPU oracle library (test infrastructure only).

``python oracle/build.py`` compiles ``oracle/dash_oracle.c`` into
``oracle/_build/libdash_oracle.so`` with gcc.  ``-ffp-contract=off`` keeps the
explicit fmaf sequence of the router restatement exactly as written, so its
block scores stay bit-identical to the CUDA router.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "dash_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libdash_oracle.so")


def build(force: bool = False) -> str:
    if (not force and os.path.exists(LIB)
            and os.path.getmtime(LIB) >= os.path.getmtime(SRC)):
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    cmd = ["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
           "-shared", "-fPIC", "-o", LIB, SRC, "-lm"]
    subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
