"""Build libvq2_b200.so (the C-ABI extension) in-tree for sm_100a with nvcc.

    python build_lib.py            # builds next to this file
The library is one translation unit (csrc/vq2_lib.cu) linked against the static CUDA runtime;
it has no torch dependency. Rebuilds only when a source is newer than the .so.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libvq2_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2", "-diag-suppress", "177"]


def sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")) + glob.glob(os.path.join(HERE, "csrc", "*.cuh"))
                  + glob.glob(os.path.join(REPO, "include", "*.h")))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and os.path.exists(LIB):
        t = os.path.getmtime(LIB)
        if all(os.path.getmtime(s) <= t for s in sources()):
            return LIB
    cmd = [NVCC, *FLAGS, os.path.join(HERE, "csrc", "vq2_lib.cu"), "-o", LIB + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
