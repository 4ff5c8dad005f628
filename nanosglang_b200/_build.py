"""Build libnsq.so (sm_100a) in-tree with nvcc.

Every ``.cu`` file under ``csrc/`` is compiled for
``-gencode arch=compute_100a,code=sm_100a`` into ``_build/`` at the repository
root and linked into ``nanosglang_b200/libnsq.so`` with the CUDA runtime
linked statically, so the library has no dependency on a driver at load time.
Runs on a machine without a GPU (nvcc cross-compiles).
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libnsq.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
              "-I" + INCLUDE, "-I" + CSRC] + ARCH


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; libnsq must be built with the CUDA toolkit")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps():
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hdrs.append(os.path.join(INCLUDE, "nsq.h"))
    return hdrs


def _stale(target: str, inputs) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(i) > t for i in inputs)


def build(verbose: bool = False, force: bool = False, jobs: int = 4) -> str:
    """Compile (if stale) and return the path of libnsq.so."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    deps = _deps()
    objs = []
    todo = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + deps):
            todo.append((s, o))

    def compile_one(so):
        s, o = so
        cmd = [nvcc] + NVCC_FLAGS + ["-c", s, "-o", o]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(s)}:\n{r.stderr}")
        return r.stderr

    if todo:
        with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
            for log in ex.map(compile_one, todo):
                if verbose and log:
                    sys.stderr.write(log)
    if force or todo or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link of libnsq.so failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
