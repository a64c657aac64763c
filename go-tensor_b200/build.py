"""Builds the native libraries of go-tensor's B200 backend in place.

* ``lib/libgotensor_cuda.so`` — the CUDA kernels and the C interface declared
  in ``include/gt_cuda.h`` (compiled for sm_100a only);
* ``lib/libgotensor_host.so`` — the C++ training-step runtime declared in
  ``include/gt_host.h``, linked against the first.

Objects are rebuilt when their source or any header is newer. Usage:
``python go-tensor_b200/build.py [-j N] [--clean]``.
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
INCLUDE = os.path.join(ROOT, "include")
CSRC = os.path.join(HERE, "csrc")
RUNTIME = os.path.join(HERE, "runtime")
BUILD = os.path.join(HERE, "lib", "obj")
LIB = os.path.join(HERE, "lib")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                     "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC, "-DGT_BUILDING_LIB"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-I", INCLUDE, "-I", os.path.join(CUDA_HOME, "include")]

CUDA_LIB = os.path.join(LIB, "libgotensor_cuda.so")
HOST_LIB = os.path.join(LIB, "libgotensor_host.so")


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


def build(jobs: int | None = None, verbose: bool = False) -> None:
    os.makedirs(BUILD, exist_ok=True)
    headers = glob.glob(os.path.join(INCLUDE, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    objs, jobs_list = [], []
    for src in cu:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if _newer(obj, [src] + headers):
            jobs_list.append([NVCC] + NVCC_FLAGS + ["-c", src, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        for out in ex.map(_run, jobs_list):
            if verbose and out.strip():
                print(out)
    if _newer(CUDA_LIB, objs):
        # Static CUDA runtime; the driver entry points are fetched at run time.
        _run([NVCC] + ARCH + ["-shared", "-o", CUDA_LIB] + objs + ["-ldl", "-lpthread"])

    host_src = sorted(glob.glob(os.path.join(RUNTIME, "*.cpp")))
    host_hdr = headers + glob.glob(os.path.join(RUNTIME, "*.hpp"))
    if host_src and (_newer(HOST_LIB, host_src + host_hdr + [CUDA_LIB])):
        _run(["g++"] + CXX_FLAGS + ["-shared", "-o", HOST_LIB] + host_src +
             ["-L", LIB, "-lgotensor_cuda", "-Wl,-rpath,$ORIGIN", "-lpthread"])


def clean() -> None:
    shutil.rmtree(LIB, ignore_errors=True)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    if a.clean:
        clean()
    build(a.j, a.v)
    print("built", CUDA_LIB, "and", HOST_LIB if os.path.exists(HOST_LIB) else "(no host runtime yet)")
    sys.exit(0)
