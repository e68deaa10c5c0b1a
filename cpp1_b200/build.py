"""Build libsmm.so in-tree with nvcc for sm_100a.

    python -m cpp1_b200.build [--force] [--verbose] [--debug-bounds]

Each .cu file under csrc/ is compiled to an object in parallel, then linked
into ``cpp1_b200/libsmm.so``.  ``--debug-bounds`` builds the bounds-checked
variant ``cpp1_b200/libsmm_debug.so`` instead (-DSMM_DEBUG_BOUNDS: every
computed offset into a structured operand is range-checked on the device;
``SMM_LIB=debug`` makes the Python binding load it).  The CUDA runtime is linked as a shared library
so the process has a single runtime instance (the one PyTorch also uses):
current-device and stream state are then shared with the caller.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OBJDIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libsmm.so")
OBJDIR_DEBUG = os.path.join(HERE, "_build_debug")
LIB_DEBUG = os.path.join(HERE, "libsmm_debug.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
    f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool, debug: bool = False) -> str:
    obj = os.path.join(OBJDIR_DEBUG if debug else OBJDIR, os.path.basename(src) + ".o")
    if _stale(obj, [src] + _headers()):
        cmd = [nvcc(), *NVCC_FLAGS, *(["-DSMM_DEBUG_BOUNDS"] if debug else []), "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr:
            print(r.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, debug_bounds: bool = False) -> str:
    objdir, lib = (OBJDIR_DEBUG, LIB_DEBUG) if debug_bounds else (OBJDIR, LIB)
    os.makedirs(objdir, exist_ok=True)
    srcs = _sources()
    if force:
        for f in os.listdir(objdir):
            os.remove(os.path.join(objdir, f))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, debug_bounds), srcs))
    if force or _stale(lib, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "shared", "-o", lib, *objs,
               "-Xlinker", "-rpath,/usr/local/cuda/lib64"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--debug-bounds", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, debug_bounds=a.debug_bounds))


if __name__ == "__main__":
    sys.exit(main())
