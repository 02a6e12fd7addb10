"""Build libcevk.so (all CUDA kernels + the C ABI) for sm_100a, in-tree.

    python rust-cev_b200/build.py [--force] [--static]

Compiles every csrc/*.cu with nvcc (relocatable device code, -O3,
-lineinfo, -gencode arch=compute_100a,code=sm_100a) in parallel into
_build/, then links rust-cev_b200/cev_b200/libcevk.so.  Rebuilds only what
changed (sources or headers newer than the objects).

``--static`` also archives rust-cev_b200/cev_b200/libcevk.a: the same
objects plus their device-link object (nvcc -dlink), so that a host linker
without nvcc (cargo's, through a build.rs) can link it; the consumer adds
-lcudart -lcuda -lstdc++.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "cev_b200", "libcevk.so")
OUT_A = os.path.join(HERE, "cev_b200", "libcevk.a")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-diag-suppress", "20044", "-I", os.path.join(ROOT, "include")]


def _headers_mtime() -> float:
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max(os.path.getmtime(h) for h in hs)


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    if not force and os.path.exists(obj) and os.path.getmtime(obj) > max(os.path.getmtime(src), _headers_mtime()):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    return obj


def _run(cmd, what):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{what} failed:\n{r.stderr}")


def build(force: bool = False, static: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(OUT) or os.path.getmtime(OUT) < newest:
        _run([NVCC, *ARCH, "-shared", "-rdc=true", *objs, "-o", OUT], "link")
    if static and (force or not os.path.exists(OUT_A) or os.path.getmtime(OUT_A) < newest):
        dlink = os.path.join(BUILD, "cevk_dlink.o")
        _run([NVCC, *ARCH, "-dlink", "-Xcompiler", "-fPIC", *objs, "-o", dlink], "device link")
        if os.path.exists(OUT_A):
            os.remove(OUT_A)
        _run(["ar", "rcs", OUT_A, *objs, dlink], "ar")
    return OUT_A if static else OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, static="--static" in sys.argv))
