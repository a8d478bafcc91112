"""Build the native parts of flb-transformer_b200 in-tree.

Outputs (next to this file, git-ignored, shipped with the source tree):
  libflb_b200.so                      C-ABI library: every CUDA kernel, compiled for sm_100a only
  wavefront_backend.<abi>.so          pybind11 module with execute_forward / execute_backward,
                                      linked against libflb_b200.so

Usage: python build.py [--force] [-j N]
Objects go to _build/ (git-ignored). Rebuilds only what changed.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")
REPO = os.path.dirname(ROOT)
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(ROOT, "_build")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

LIB_NAME = "libflb_b200.so"
CU_SOURCES = [
    "c_abi.cu",
    "attention_generic.cu",
    "attention_fast.cu",
    "wavefront_prims.cu",
    "wavefront_grid.cu",
    "flb_block.cu",
    "microbench.cu",
    "umma_selftest.cu",
]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",  # export only the C API declared in include/flb_b200.h
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
    "-I", INCLUDE,
]


def _headers():
    out = [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    out += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return out


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout)
        raise RuntimeError("build step failed: " + " ".join(cmd[:6]) + " ...")
    if r.stdout.strip():
        # keep ptxas spill warnings visible
        sys.stderr.write(r.stdout)


def build_library(force: bool = False, jobs: int = 8) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = _headers()
    objs = []
    todo = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + headers):
            todo.append([NVCC, *NVCC_FLAGS, "-c", s, "-o", o])
    if todo:
        with ThreadPoolExecutor(max_workers=jobs) as ex:
            list(ex.map(_run, todo))
    lib = os.path.join(ROOT, LIB_NAME)
    if force or todo or _stale(lib, objs):
        _run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
              "-o", lib, *objs, "-lcublas",
              "-Xlinker", "-rpath," + os.path.join(CUDA_HOME, "lib64")])
    return lib


def build_backend(force: bool = False) -> str:
    import torch.utils.cpp_extension as ce  # deferred: torch import is slow
    import pybind11

    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    out = os.path.join(ROOT, "wavefront_backend" + suffix)
    src = os.path.join(CSRC, "wavefront_backend.cpp")
    lib = os.path.join(ROOT, LIB_NAME)
    if not force and not _stale(out, [src, lib] + _headers()):
        return out
    incs = ce.include_paths() + [pybind11.get_include(), sysconfig.get_paths()["include"],
                                 INCLUDE, os.path.join(CUDA_HOME, "include")]
    libdirs = ce.library_paths()
    import torch
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O3", "-std=c++17", "-shared", "-fPIC", src, "-o", out,
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=wavefront_backend",
           "-DTORCH_API_INCLUDE_EXTENSION_H"]
    cmd += [f"-I{p}" for p in incs]
    cmd += [f"-L{p}" for p in libdirs] + [f"-L{ROOT}"]
    cmd += ["-lflb_b200", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda",
            "-ltorch_cuda"]
    cmd += ["-Wl,-rpath,$ORIGIN"] + [f"-Wl,-rpath,{p}" for p in libdirs]
    _run(cmd)
    return out


def build(force: bool = False, jobs: int = 8) -> None:
    build_library(force=force, jobs=jobs)
    build_backend(force=force)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    a = ap.parse_args()
    build(force=a.force, jobs=a.j)
    print("built", os.path.join(ROOT, LIB_NAME))
