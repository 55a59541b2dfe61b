"""Builds libp0mm.so (the C-ABI library: every CUDA kernel of this package) in-tree for sm_100a with nvcc.

python -m p0pc0rn_b200.build      # or p0pc0rn_b200.build.build()
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libp0mm.so")
SOURCES = ["context.cu", "gemv.cu", "gemm.cu", "pack.cu"]
HEADERS = ["internal.h", "tc.cuh", os.path.join("..", "..", "include", "p0mm.h")]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.sep not in c or os.path.exists(c)):
            return c
    return "nvcc"


def _stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, s) for s in SOURCES + HEADERS] + [__file__]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, ptxas_v=False):
    """Compile every .cu under csrc/ into libp0mm.so (skipped when up to date)."""
    if not force and not _stale():
        return LIB
    host_cc = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-ccbin", host_cc,
           "-o", LIB + ".tmp"] + [os.path.join(CSRC, s) for s in SOURCES]
    if ptxas_v:
        cmd.insert(1, "-Xptxas=-v")
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    if verbose or ptxas_v:
        print(r.stdout + r.stderr, file=sys.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_v="-v" in sys.argv)
    print(LIB)
