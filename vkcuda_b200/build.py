"""Build libVCRuntime.so (the runtime plus every sm_100a kernel) in-tree.

    python -m vkcuda_b200.build            # incremental
    python -m vkcuda_b200.build --force    # rebuild everything

Each source in csrc/ is compiled by nvcc for sm_100a (`-gencode
arch=compute_100a,code=sm_100a`) into vkcuda_b200/_build/, then linked into
vkcuda_b200/lib/libVCRuntime.so with the CUDA runtime linked statically (the
driver API is reached through cudaGetDriverEntryPointByVersion, so the library
loads on machines without a GPU driver and exports every symbol of
include/vc_b200.h and include/vc/Runtime/VCRuntime.h).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libVCRuntime.so")

SOURCES = [
    "runtime.cpp",
    "stream_kernels.cu",
    "gemm_tcgen05.cu",
    "gemm_f32_tcgen05.cu",
    "gemm_simt.cu",
    "flash_fwd_tcgen05.cu",
    "flash_fwd_f32.cu",
    "selftest.cu",
]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
          "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libVCRuntime")


def _headers_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    paths += [os.path.join(ROOT, "include", "vc_b200.h"),
              os.path.join(ROOT, "include", "vc", "Runtime", "VCRuntime.h")]
    return max(os.path.getmtime(p) for p in paths)


def _compile(src: str, force: bool, verbose_ptxas: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    if (not force and os.path.exists(obj)
            and os.path.getmtime(obj) >= max(os.path.getmtime(path), _headers_mtime())):
        return obj
    cmd = [nvcc(), *ARCH, *COMMON, "-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd[1:1] = ["-x", "cu"]
    if verbose_ptxas and src.endswith(".cu"):
        cmd.append("-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
    if verbose_ptxas and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    """Compile and link; returns the path of libVCRuntime.so."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose_ptxas), SOURCES))
    if (force or not os.path.exists(LIB)
            or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static",
               "-Xcompiler", "-fPIC", "-lpthread", "-ldl", "-lrt"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / smem usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.ptxas_v))
