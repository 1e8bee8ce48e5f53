"""Build libhyperion_mlx.so (the engine + kernels) for sm_100a, in-tree.

nvcc cross-compiles without a GPU, so this runs anywhere CUDA 12.9 is installed.
The library links only the CUDA runtime; it has no Python or torch dependency.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libhyperion_mlx.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-Wall,-Wuninitialized", "--expt-relaxed-constexpr",
         "-I", os.path.join(REPO, "include"), "-I", CSRC]
SOURCES = ["qmv.cu", "qmv_packed.cu", "qmv_batched.cu", "qmm.cu", "attention.cu", "attention_fused.cu", "attention_tc.cu", "tma_host.cu", "qmm_tc.cu", "tp.cu", "elementwise.cu", "sampler.cu", "engine.cu", "abi.cu", "ops_abi.cu",
           "geometry.cc", "safetensors.cc"]


def _obj(src: str) -> str:
    return os.path.join(BUILD, os.path.splitext(src)[0] + ".o")


def _headers_mtime() -> float:
    m = 0.0
    for d in (CSRC, os.path.join(REPO, "include")):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh")):
                m = max(m, os.path.getmtime(os.path.join(d, f)))
    return m


def _compile(src: str, extra: list[str]) -> str:
    out = _obj(src)
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", out]
    if src.endswith(".cc"):
        cmd = [NVCC, *FLAGS, *extra, "-x", "cu", "-c", os.path.join(CSRC, src), "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return out


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdr = _headers_mtime()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    todo = []
    for s in SOURCES:
        o = _obj(s)
        if force or verbose_ptxas or not os.path.exists(o) or os.path.getmtime(o) < max(
                os.path.getmtime(os.path.join(CSRC, s)), hdr):
            todo.append(s)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(lambda s: _compile(s, extra), todo))
    objs = [_obj(s) for s in SOURCES]
    if force or todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB + ".tmp", *objs, "-lcudart", "-lcuda", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="--ptxas" in sys.argv))
