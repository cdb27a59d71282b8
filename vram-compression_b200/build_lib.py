"""Build librans_b200.so in-tree with nvcc for sm_100a (B200).

    python vram-compression_b200/build_lib.py [--force]

The library is compiled from csrc/*.cu and csrc/*.cpp with explicit
`-gencode arch=compute_100a,code=sm_100a`; nothing is JIT-compiled at import
time on the GPU box, the prebuilt .so travels with the source tree.
"""
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "librans_b200.so")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def stale(lib=LIB):
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return any(os.path.getmtime(s) > t for s in deps)


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found: cannot build librans_b200.so")
    return exe


def build(force=False, verbose=False, extra=()):
    if not force and not stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), "-O3", ARCH, "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O3",
           "-I", INCLUDE, "-o", tmp, *extra, *sources(), "-lpthread"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.check_call(cmd)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else [])
    print(LIB)
