"""Build the sm_100a C-ABI library libdfsnn_b200.so in-tree.

    python df-snn-official_b200/build.py [--verbose]

Compiles every csrc/*.cu with nvcc for sm_100a (-gencode arch=compute_100a,code=sm_100a)
into df-snn-official_b200/dfsnn_b200/_lib/libdfsnn_b200.so, which the Python package loads
with ctypes.  The CUDA runtime is linked statically, so the library only needs the driver.
Rebuilds only when a source or header is newer than the library.
"""
import argparse
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "dfsnn_b200", "_lib")
LIB = os.path.join(OUT_DIR, "libdfsnn_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return sources() + sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
                              + glob.glob(os.path.join(REPO, "include", "*.h")))


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in _deps())


def nvcc():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def build(verbose=False, force=False, jobs=None):
    if not force and up_to_date():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    obj_dir = os.path.join(HERE, "_build")
    os.makedirs(obj_dir, exist_ok=True)
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-ccbin", "g++",
                    "-I", os.path.join(REPO, "include")]
    if verbose:
        flags += ["-Xptxas", "-v"]
    procs = []
    objs = []
    for src in sources():
        obj = os.path.join(obj_dir, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        procs.append(subprocess.Popen([nvcc(), *flags, "-c", src, "-o", obj]))
    bad = [p for p in procs if p.wait() != 0]
    if bad:
        raise RuntimeError("nvcc failed")
    tmp = LIB + ".tmp"
    subprocess.check_call([nvcc(), *ARCH, "-shared", "-o", tmp, *objs])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(verbose=args.verbose, force=args.force or args.verbose))
    sys.exit(0)
