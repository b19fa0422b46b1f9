"""Build the oracle's C restatement (test infrastructure; see oracle.py).

``python -m oracle.build`` or ``oracle.build.build()`` compiles
``rq_oracle.c`` into ``oracle/_build/librq_oracle.so`` with gcc, strict IEEE
arithmetic (no fast-math, no FMA contraction) so that it reproduces torch's
CPU results bit for bit.
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "rq_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
OUT = os.path.join(OUT_DIR, "librq_oracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = OUT + f".tmp{os.getpid()}"
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-fno-fast-math",
           "-ffp-contract=off", "-Wall", "-o", tmp, SRC, "-lm"]
    subprocess.check_call(cmd)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force=True))
