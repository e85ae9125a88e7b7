"""Build libholmes_cuda.so in-tree (nvcc, sm_100a only).

    python -m holmes_b200.build          # incremental
    python -m holmes_b200.build --force  # rebuild everything

The library lands in ``holmes_b200/lib/libholmes_cuda.so``; it is git-ignored but travels with the
working tree, so a GPU host uses exactly what was built here.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "lib", "obj")
LIB = os.path.join(HERE, "lib", "libholmes_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-Xcompiler",
         "-O2", "-Xptxas", "-warn-spills"]
SOURCES = ["context.cu", "nttk.cu", "misc.cu", "mac_tc.cu", "capi.cu", "noalloc.cu", "peer.cu"]


def _deps() -> list[str]:
    names = [f for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return [os.path.join(CSRC, f) for f in names] + [os.path.join(os.path.dirname(HERE), "include", "holmes_cuda.h")]


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _compile(src: str, force: bool, extra: list[str]) -> str:
    obj = os.path.join(OBJ, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    if force or _stale(obj, [path] + _deps()):
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", path, "-o", obj + ".tmp"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
        if res.stderr.strip():
            sys.stderr.write(res.stderr)
        os.replace(obj + ".tmp", obj)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False, defines=(), out: str | None = None) -> str:
    """Compile every source and link ``out`` (default ``lib/libholmes_cuda.so``); ``defines`` are extra -D flags
    for a variant build, which then gets its own object directory."""
    global OBJ
    obj_dir = OBJ if not defines else OBJ + "_" + "_".join(d.replace("=", "") for d in defines)
    target = LIB if out is None else out
    os.makedirs(obj_dir, exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    extra += [f"-D{d}" for d in defines]
    saved, OBJ = OBJ, obj_dir
    try:
        with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
            objs = list(ex.map(lambda s: _compile(s, force, extra), SOURCES))
    finally:
        OBJ = saved
    if force or _stale(target, objs):
        tmp = target + f".{os.getpid()}.tmp"
        cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, target)
    return target


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="--ptxas" in sys.argv))
