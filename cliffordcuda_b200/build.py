"""Build the native library in-tree: ``python -m cliffordcuda_b200.build``.

Runs the Makefile in ``csrc/`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``);
nvcc cross-compiles without a GPU.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(jobs=None, verbose=False):
    jobs = jobs or max(1, os.cpu_count() or 1)
    cmd = ["make", "-C", os.path.join(HERE, "csrc"), f"-j{jobs}"]
    subprocess.run(cmd, check=True, stdout=None if verbose else subprocess.DEVNULL)
    return os.path.join(HERE, "libcliffordcuda_b200.so")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
