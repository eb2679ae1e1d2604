"""Build the oracle's C restatement (oracle/_build/libquant_ref.so) with gcc - TEST INFRASTRUCTURE.

Plain -O2 without fast-math, so float32 division and rintf keep IEEE round-to-nearest-even semantics.
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "quant_ref.c")
LIB = os.path.join(HERE, "_build", "libquant_ref.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    subprocess.run(["gcc", "-O2", "-fno-fast-math", "-ffp-contract=off", "-shared", "-fPIC", SRC, "-o", LIB, "-lm"],
                   check=True)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
