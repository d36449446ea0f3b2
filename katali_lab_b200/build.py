"""Build libkatali_cuda.so (the plugin) and libkatali_cuda_loader.so (the dlopen shim).

nvcc cross-compiles for sm_100a only; no GPU is needed to build. The CUDA
runtime is linked statically, so the plugin needs only the NVIDIA driver at run
time, like the reference's katali_cuda.dll.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = os.path.join(PKG, "lib")
PLUGIN = os.path.join(LIBDIR, "libkatali_cuda.so")
LOADER = os.path.join(LIBDIR, "libkatali_cuda_loader.so")
CHECK = os.path.join(LIBDIR, "katali_cuda_check")  # command-line checks (cuda-info / cuda-check ...)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = srcs + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) \
        + glob.glob(os.path.join(INCLUDE, "*.h"))
    if force or _stale(PLUGIN, deps):
        cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared",
               "-Xcompiler", "-fPIC", "-Xptxas", "-v" if verbose else "-O3",
               "-I", INCLUDE, "-I", CSRC, "-o", PLUGIN, *srcs, "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc failed")
        if verbose:
            sys.stderr.write(r.stderr)
    loader_src = os.path.join(CSRC, "loader", "katali_cuda_loader.c")
    cc = os.environ.get("CC", "gcc")
    if os.path.exists(loader_src) and (force or _stale(LOADER, [loader_src] + deps)):
        subprocess.run([cc, "-std=c11", "-O2", "-fPIC", "-shared", "-Wall", "-I", INCLUDE,
                        "-o", LOADER, loader_src, "-ldl"], check=True)
    check_src = os.path.join(CSRC, "loader", "katali_cuda_check.c")
    if os.path.exists(check_src) and (force or _stale(CHECK, [check_src, LOADER] + deps)):
        subprocess.run([cc, "-std=c11", "-O2", "-Wall", "-I", INCLUDE, "-o", CHECK, check_src,
                        "-L", LIBDIR, "-lkatali_cuda_loader", "-Wl,-rpath,$ORIGIN", "-lm"],
                       check=True)
    return PLUGIN


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(PLUGIN)
