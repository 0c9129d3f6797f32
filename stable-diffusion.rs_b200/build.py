"""Build libsdq.so in-tree with nvcc for sm_100a (B200).

    python stable-diffusion.rs_b200/build.py [--force] [--verbose]

Each ``csrc/*.cu`` is compiled separately (no relocatable device code: every
``__device__`` symbol lives in the one file that uses it) and linked into
``stable-diffusion.rs_b200/libsdq.so`` next to this script, where the built
library travels with the source tree.  The CUDA runtime is linked statically,
so the library's only dynamic dependencies are libc / libstdc++ and NCCL.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libsdq.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-v,-warn-spills", "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for c in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def nccl_paths():
    """(include dir, lib dir) of an NCCL with headers: the system one first."""
    cands = [("/usr/include", "/usr/lib/x86_64-linux-gnu")]
    try:
        import nvidia.nccl as nn  # type: ignore
        base = list(nn.__path__)[0]
        cands.append((os.path.join(base, "include"), os.path.join(base, "lib")))
    except Exception:
        pass
    for inc, lib in cands:
        if os.path.exists(os.path.join(inc, "nccl.h")) and any(
                f.startswith("libnccl.so") for f in os.listdir(lib) if os.path.isdir(lib)):
            return inc, lib
    raise RuntimeError("NCCL headers / library not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(ROOT, "include", "sdq.h"))
    return hs


def stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cc = nvcc()
    inc, libdir = nccl_paths()
    objs = []
    hdrs = headers()
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or stale(obj, [src] + hdrs):
            cmd = [cc, *ARCH, *NVCC_FLAGS, "-I", inc, "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            res = subprocess.run(cmd, capture_output=True, text=True)
            if verbose or res.returncode != 0:
                sys.stdout.write(res.stdout)
                sys.stderr.write(res.stderr)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src}")
    if force or stale(LIB, objs):
        cmd = [cc, *ARCH, "-shared", "-o", LIB, *objs, "-L", libdir, "-lnccl",
               "-Xlinker", "-rpath", "-Xlinker", libdir]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
