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
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = os.path.join(PKG, "lib")
PLUGIN = os.path.join(LIBDIR, "libkatali_cuda.so")
LOADER = os.path.join(LIBDIR, "libkatali_cuda_loader.so")
CHECK = os.path.join(LIBDIR, "katali_cuda_check")  # command-line checks (cuda-info / cuda-check ...)
OBJDIR = os.path.join(LIBDIR, "obj")

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


def _compile(src: str, obj: str, verbose: bool) -> str:
    cmd = [_nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-c", "-Xcompiler", "-fPIC",
           "-Xptxas", "-v" if verbose else "-O3", "-I", INCLUDE, "-I", CSRC, "-o", obj, src]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}{r.stderr}")
    return r.stderr if verbose else ""


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every csrc/*.cu to an object (in parallel, only the stale ones), link the
    plugin, then the loader and the check CLI."""
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) \
        + glob.glob(os.path.join(INCLUDE, "*.h"))
    deps = srcs + headers
    objs = [os.path.join(OBJDIR, os.path.basename(s)[:-3] + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(o, [s] + headers)]
    if todo:
        with ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            for log in ex.map(lambda so: _compile(so[0], so[1], verbose), todo):
                if log:
                    sys.stderr.write(log)
    if force or todo or _stale(PLUGIN, objs):
        cmd = [_nvcc(), *ARCH, "--shared", "-Xcompiler", "-fPIC", "-o", PLUGIN, *objs, "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc link failed")
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
