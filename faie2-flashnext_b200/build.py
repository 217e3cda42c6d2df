"""Build libfaie2fn.so (the engine's C ABI) from csrc/*.cu for sm_100a, in-tree under lib/.

Each translation unit is compiled separately (in parallel), then linked into one shared library with the CUDA
runtime linked statically, so the library needs only the NVIDIA driver at run time.

usage: python build.py [--force] [--jobs N] [--debug]
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")  # the C ABI header (include/faie2fn.h)
OBJ = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libfaie2fn.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++20", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
                  glob.glob(os.path.join(INCLUDE, "*.h")))


def stale(target, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def compile_one(src, extra):
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if not stale(obj, [src, *headers(), __file__]) and not extra.get("force"):
        return obj, None
    cmd = [nvcc(), *ARCH, *FLAGS, *extra.get("flags", []), "-I", CSRC, "-I", INCLUDE, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return None, f"$ {' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    return obj, (r.stderr.strip() or None)


def build(force: bool = False, jobs: int | None = None, debug: bool = False, verbose: bool = True) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    extra = {"force": force, "flags": ["-DFN_DEBUG=1"] if debug else []}
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(len(srcs), os.cpu_count() or 4)) as ex:
        res = list(ex.map(lambda s: compile_one(s, extra), srcs))
    errs = [msg for obj, msg in res if obj is None]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    if verbose:
        for (obj, msg), s in zip(res, srcs):
            if msg:
                print(f"[{os.path.basename(s)}]\n{msg}", file=sys.stderr)
    objs = [o for o, _ in res]
    if force or stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", LIB, *objs, "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n$ {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--debug", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.debug))
