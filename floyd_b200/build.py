"""Builds the sm_100a CUDA library of the verify-step backend in-tree.

    python -m floyd_b200.build        ->  floyd_b200/libfloyd_cuda.so

nvcc compiles for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`);
the library has no other code path.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libfloyd_cuda.so")
SOURCES = [os.path.join(HERE, "csrc", "runtime.cu")]
DEPS = SOURCES + [os.path.join(HERE, "csrc", f) for f in os.listdir(os.path.join(HERE, "csrc"))] + [
    os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in DEPS if os.path.exists(p))


def build(force=False, verbose=False):
    if not force and not needs_build():
        return LIB
    cmd = [nvcc(), "-O3", "-std=c++17", "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
           "-gencode", "arch=compute_100a,code=sm_100a", "--expt-relaxed-constexpr",
           "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp"] + SOURCES + ["-lcudart"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
