"""Build libquantpack_b200.so in-tree with nvcc for sm_100a (no torch headers: the library is a plain C ABI).

    python -m vllm_quantpack_b200.build [--force] [--verbose]

Each .cu under csrc/ compiles to an object with relocatable device code (the device error word is shared across
files), then nvcc links them into one shared library next to this file. ptxas register / spill reports are kept in
_build/*.ptxas.txt.
"""
import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libquantpack_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
              "--expt-relaxed-constexpr"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the quantpack_b200 kernels need the CUDA toolkit to build")
    return path


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps():
    return sources() + sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h")))


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _deps() + [os.path.abspath(__file__)])


def _compile(src, extra):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc()] + ARCH + NVCC_FLAGS + list(extra) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stderr[-6000:]}")
    with open(os.path.join(BUILD, os.path.basename(src)[:-3] + ".ptxas.txt"), "w") as fh:
        fh.write(r.stderr)
    return obj


def build(force=False, verbose=False, extra=()):
    """Compile every kernel for sm_100a and link the shared library. Returns its path."""
    if not force and up_to_date():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), srcs))
    tmp = LIB + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-rdc=true", "-Xcompiler", "-fPIC", "-o", tmp] + objs + ["-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stderr[-4000:]}")
    os.replace(tmp, LIB)
    if verbose:
        for s in srcs:
            print(open(os.path.join(BUILD, os.path.basename(s)[:-3] + ".ptxas.txt")).read())
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
