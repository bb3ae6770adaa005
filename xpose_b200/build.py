"""Build libxp_cuda.so in-tree with nvcc for sm_100a (and the test oracles).

    python -m xpose_b200.build
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libxp_cuda.so")
SRC = os.path.join(HERE, "csrc", "xp_cuda.cu")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc")

NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-shared",
    "-diag-suppress", "1886,842",
]


def _sources():
    d = os.path.join(HERE, "csrc")
    return [os.path.join(d, f) for f in os.listdir(d)] + [os.path.join(ROOT, "include", "xp_cuda.h")]


def _stale(out, srcs):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs)


def build_cuda(force=False, verbose=False):
    if not force and not _stale(LIB, _sources()):
        return LIB
    cmd = [NVCC, *NVCC_FLAGS, "-o", LIB, SRC]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return LIB


def build_oracle(verbose=False):
    """The CPU checkers (test infrastructure): oracle/liboracle.so always,
    oracle/_ref/libxpref.so when the reference tree is present."""
    env = dict(os.environ)
    env.pop("CC", None)
    env.pop("CXX", None)
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True, env=env,
                   stdout=None if verbose else subprocess.DEVNULL)


def main():
    build_cuda(force="--force" in sys.argv, verbose=True)
    build_oracle(verbose=True)
    print("built", LIB)


if __name__ == "__main__":
    main()
