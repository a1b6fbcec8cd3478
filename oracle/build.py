"""Build the CPU oracle (test infrastructure only) into oracle/liboracle.so.

The reference (rtburger/grout) is Rust + cuTile and cannot be compiled here
(no rustc/cargo, no cutile crates, no tileiras), so there is no oracle/_ref
build; the oracle is the C++ restatement in oracle.cpp.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "oracle.cpp")
OUT = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    # -march=x86-64-v2: portable to the GPU box's host CPU (same image, maybe
    # a different CPU model); -ffp-contract=off keeps the bit-exact norm/RoPE
    # restatement free of FMA contraction.
    cmd = ["g++", "-O3", "-march=x86-64-v2", "-fopenmp", "-ffp-contract=off",
           "-fno-fast-math", "-shared", "-fPIC", "-o", OUT + ".tmp", SRC]
    subprocess.check_call(cmd)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
