"""Compile the oracle's C restatement into ``oracle/liboracle.so``.

TEST INFRASTRUCTURE ONLY.  The reference has no C/C++/CUDA source on this
path (its arithmetic is MLX, not vendored; the Swift repacker needs a Swift
toolchain that is absent), so there is no ``oracle/_ref`` build: the oracle
restatement is both the checker and the timed CPU baseline (kind "port").

router_ref.c is compiled with -ffp-contract=off: its float32 evaluation order
is part of the contract with the device router kernel.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    srcs = [os.path.join(HERE, "c", n) for n in ("router_ref.c", "moe_ref.c", "synth_ref.c")]
    if not force and os.path.exists(LIB) and all(os.path.getmtime(LIB) >= os.path.getmtime(s) for s in srcs):
        return LIB
    tmp = os.path.join(HERE, "_build")
    os.makedirs(tmp, exist_ok=True)
    objs = []
    flags = {
        "router_ref.c": ["-O2", "-ffp-contract=off", "-fno-fast-math", "-mfma", "-fopenmp"],
        "moe_ref.c": ["-O3", "-mavx2", "-mfma", "-ffast-math", "-fopenmp"],
        "synth_ref.c": ["-O3", "-ffp-contract=off", "-fno-fast-math", "-fopenmp"],
    }
    for s in srcs:
        o = os.path.join(tmp, os.path.basename(s) + ".o")
        subprocess.check_call(["gcc", "-std=c11", "-fPIC", "-c", s, "-o", o] + flags[os.path.basename(s)])
        objs.append(o)
    subprocess.check_call(["gcc", "-shared", "-o", LIB] + objs + ["-fopenmp", "-lm"])
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
