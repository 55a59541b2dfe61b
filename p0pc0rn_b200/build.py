"""Builds libp0mm.so (the C-ABI library: every CUDA kernel of this package) in-tree for sm_100a with nvcc.

python -m p0pc0rn_b200.build      # or p0pc0rn_b200.build.build()
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libp0mm.so")
SOURCES = ["context.cu", "gemv.cu", "gemv_v3.cu", "gemv_v4.cu", "gemv_v5.cu", "chain.cu", "gemm.cu", "pack.cu", "lops.cu", "io.cu"]
HEADERS = ["internal.h", "tc.cuh", "gemv_common.cuh", os.path.join("..", "..", "include", "p0mm.h")]
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
    common = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-ccbin", host_cc]
    if ptxas_v:
        common.insert(1, "-Xptxas=-v")
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = [os.path.join(objdir, os.path.splitext(s)[0] + ".o") for s in SOURCES]
    cmds = [common + ["-c", os.path.join(CSRC, s), "-o", o] for s, o in zip(SOURCES, objs)]
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=len(cmds)) as ex:      # one nvcc per translation unit, in parallel
        results = list(ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), cmds))
    for c, r in zip(cmds, results):
        if verbose:
            print(" ".join(c), file=sys.stderr)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
        if verbose or ptxas_v:
            print(r.stdout + r.stderr, file=sys.stderr)
    link = [nvcc(), *ARCH, "-shared", "-ccbin", host_cc, "-o", LIB + ".tmp"] + objs
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + r.stdout + r.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_v="-v" in sys.argv)
    print(LIB)
