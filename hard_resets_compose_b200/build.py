"""Build liblifb.so (the C-ABI CUDA library) in-tree for sm_100a.

    python -m hard_resets_compose_b200.build      # or build() from Python

nvcc compiles every csrc/*.cu for `-gencode arch=compute_100a,code=sm_100a`
and links them into hard_resets_compose_b200/lib/liblifb.so.  The build runs
on a machine without a GPU (nvcc cross-compiles); the .so travels with the
source tree to the GPU machine.  Rebuilds only when a source is newer.
"""
from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "liblifb.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-Wall", "-I", CSRC, "-I", INCLUDE]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin directory on PATH")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, defines=(), out: str = None) -> str:
    """Compile liblifb.so.  `defines` are extra -D flags (the build-time
    tunables of csrc/chunk_tma.cu); `out` builds to another path instead of
    the in-tree library."""
    target = out or LIB
    if out is None and not force and not _stale():
        return LIB
    libdir = os.path.dirname(target)
    os.makedirs(libdir, exist_ok=True)
    objdir = os.path.join(libdir, "obj" if out is None else "obj_" + os.path.basename(target))
    os.makedirs(objdir, exist_ok=True)
    nvcc = _nvcc()
    objs, cmds = [], []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        cmds.append([nvcc, *ARCH, *NVCC_FLAGS, *[f"-D{d}" for d in defines], "-c", src, "-o", obj])
        objs.append(obj)
    # one nvcc per translation unit, as many at once as there are cores
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        for cmd, res in zip(cmds, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), cmds)):
            if verbose:
                print(" ".join(cmd))
            if res.stdout or res.stderr:
                print(res.stdout + res.stderr, end="", file=sys.stderr)
            if res.returncode:
                raise subprocess.CalledProcessError(res.returncode, cmd, res.stdout, res.stderr)
    tmp = target + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, target)
    return target


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
