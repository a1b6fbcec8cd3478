"""Builds libgrout_attn.so in-tree with nvcc for sm_100a.

    python -m grout_b200.build [--force]

One object per .cu file under csrc/, linked into grout_b200/libgrout_attn.so
(static CUDA runtime, so the library carries no dependency beyond the
driver).  The build is skipped when the library is newer than every source.
"""
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libgrout_attn.so")
BUILD_DIR = os.path.join(HERE, "_build")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-I" + os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(
        os.path.join(CSRC, "*.h")) + [os.path.join(ROOT, "include", "grout_attn.h"), __file__]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(force: bool = False, verbose: bool = False, extra_flags=()) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = []
    procs = []
    for src in _sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc(), *NVCC_FLAGS, *extra_flags, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        procs.append((subprocess.Popen(cmd), cmd))
        objs.append(obj)
    for p, cmd in procs:
        if p.wait() != 0:
            raise RuntimeError("nvcc failed: " + " ".join(cmd))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs]
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else []
    print(build(force="--force" in sys.argv or bool(extra), verbose=v, extra_flags=extra))
