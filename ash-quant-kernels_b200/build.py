"""Build the in-tree native libraries of ashqk-b200.

Produces, next to the Python package (``ashqk/``):

* ``libashqk_b200.so`` -- the CUDA kernels and the C ABI of
  ``include/ashqk_b200.h``, compiled by nvcc for sm_100a only, CUDA runtime
  linked statically, no PyTorch dependency;
* ``_ashqk_torch.so`` -- the thin PyTorch operator binding
  (``torch.ops.ashqk.*``), linked against the library above with an
  ``$ORIGIN`` rpath.

Usage: ``python ash-quant-kernels_b200/build.py [--force] [-j N]``. Rebuilds only
what is older than its sources.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "ashqk")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(PKG, "libashqk_b200.so")
TORCH_LIB = os.path.join(PKG, "_ashqk_torch.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-rdc=true", "-I", INCLUDE, "-I", CSRC]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda_home, "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")


def build_cuda_library(force: bool = False, jobs: int = 8) -> str:
    os.makedirs(OBJ, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    objs = []
    jobs_list = []
    for src in sources:
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            jobs_list.append([_nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for fut in [ex.submit(_run, c) for c in jobs_list]:
            fut.result()
    if force or _stale(LIB, objs):
        _run([_nvcc(), *ARCH, "-shared", "-rdc=true", "-cudart", "static", "-o", LIB, *objs])
    return LIB


def build_torch_binding(force: bool = False) -> str:
    src = os.path.join(CSRC, "torch_binding.cpp")
    if not (force or _stale(TORCH_LIB, [src, LIB, os.path.join(INCLUDE, "ashqk_b200.h")])):
        return TORCH_LIB
    import torch
    from torch.utils import cpp_extension

    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = [f"-I{p}" for p in cpp_extension.include_paths()] + [f"-I{cuda_home}/include", f"-I{INCLUDE}"]
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_ashqk_torch", *inc, src,
           "-o", TORCH_LIB, f"-L{PKG}", "-lashqk_b200", f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch_cpu",
           "-ltorch_cuda", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    _run(cmd)
    return TORCH_LIB


def build(force: bool = False, jobs: int = 8) -> None:
    build_cuda_library(force, jobs)
    build_torch_binding(force)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=os.cpu_count() or 8)
    ns = ap.parse_args()
    build(ns.force, ns.jobs)
    print("built", LIB, TORCH_LIB)
