"""Builds libqkv.so (kernels + engine + C ABI) in-tree for sm_100a.

    python -m qwfn_hybrid_b200.build             # incremental
    python -m qwfn_hybrid_b200.build --force     # from scratch
    python -m qwfn_hybrid_b200.build --timeline  # libqkv_timeline.so, phase-stamped (analysis only)

nvcc cross-compiles for sm_100a without a GPU.  Objects go to qwfn_hybrid_b200/_build/, the
shared library to qwfn_hybrid_b200/libqkv.so (git-ignored, shipped to the GPU box with the
tree).  The CUDA runtime is linked statically so the library needs only the driver.  The timeline
build compiles the same sources with -DQKV_TIMELINE (per-CTA %globaltimer stamps of the decode,
merge and projection kernels, read by qwfn_hybrid_b200.timeline) into _build_tl/ and
libqkv_timeline.so; the product never loads it.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libqkv.so")
OBJ_TL = os.path.join(HERE, "_build_tl")
LIB_TL = os.path.join(HERE, "libqkv_timeline.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-Wall,-Wextra", "-I", os.path.join(ROOT, "include"),
          "-I", CSRC, "--expt-relaxed-constexpr"]
HEADERS = [os.path.join(ROOT, "include", "qkv.h")] + [
    os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, extra: list[str], obj_dir: str = OBJ) -> str:
    obj = os.path.join(obj_dir, os.path.basename(src) + ".o")
    if _stale(obj, [src] + HEADERS):
        cmd = [NVCC, *ARCH, *COMMON, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False, timeline: bool = False) -> str:
    obj_dir, lib = (OBJ_TL, LIB_TL) if timeline else (OBJ, LIB)
    os.makedirs(obj_dir, exist_ok=True)
    if force:
        for f in os.listdir(obj_dir):
            os.remove(os.path.join(obj_dir, f))
    extra = (["-Xptxas", "-v"] if verbose_ptxas else []) + (["-DQKV_TIMELINE"] if timeline else [])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, obj_dir), sources()))
    if force or _stale(lib, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", lib, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="--ptxas" in sys.argv, timeline="--timeline" in sys.argv))
