"""Builds liblarder_b200.so in-tree with nvcc for sm_100a (B200).

    python -m larder_b200.build [--force]

One translation unit (csrc/lb2.cu includes every kernel header), linked against the static CUDA runtime, so the
.so carries no dependency beyond the driver and travels with the repository.
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
OUT = os.path.join(HERE, "liblarder_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
         "-shared", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def sources():
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")) + glob.glob(os.path.join(HERE, "csrc", "*.cuh"))
                  + [os.path.join(ROOT, "include", "larder_b200.h")])


def stale():
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    return any(os.path.getmtime(s) > t for s in sources())


def build(force=False, verbose=False):
    if not force and not stale():
        return OUT
    cmd = [NVCC, *FLAGS, "-o", OUT + ".tmp", os.path.join(HERE, "csrc", "lb2.cu")]
    if verbose:
        cmd.insert(-3, "-Xptxas")
        cmd.insert(-3, "-v")
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
