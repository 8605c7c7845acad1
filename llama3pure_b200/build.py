"""Compile libllama3pure_attn.so in-tree for sm_100a with nvcc.

The library is plain C ABI (include/llama3pure_attn.h) over CUDA kernels in
llama3pure_b200/csrc/.  It is built next to this file so it travels with the
repository; nothing is installed into site-packages.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import tempfile

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
INCLUDE = os.path.join(ROOT, "include")
CSRC = os.path.join(PKG, "csrc")
LIB_NAME = "libllama3pure_attn.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libllama3pure_attn.so")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) +
                  glob.glob(os.path.join(INCLUDE, "*.h")))


def up_to_date(out: str = LIB_PATH) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose: bool = False, out: str = LIB_PATH, extra: list[str] | None = None) -> str:
    """Build the shared library if any source is newer; return its path.  The
    translation units compile in parallel into a temporary directory, then
    link into `out`."""
    if not force and up_to_date(out):
        return out
    units = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    flags = [*ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
             "-I", INCLUDE, "-I", CSRC, *(extra or [])]
    with tempfile.TemporaryDirectory() as tmp:
        objs, procs = [], []
        for u in units:
            obj = os.path.join(tmp, os.path.basename(u) + ".o")
            cmd = [nvcc(), *flags, "-c", u, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            procs.append(subprocess.Popen(cmd))
            objs.append(obj)
        failed = [u for u, p in zip(units, procs) if p.wait() != 0]
        if failed:
            raise subprocess.CalledProcessError(1, f"nvcc -c {' '.join(failed)}")
        link = [nvcc(), *ARCH_FLAGS, "-shared", "-o", out + ".tmp", *objs]
        if verbose:
            print(" ".join(link), flush=True)
        subprocess.run(link, check=True)
    os.replace(out + ".tmp", out)
    return out


if __name__ == "__main__":
    print(build(force=True, verbose=True))
