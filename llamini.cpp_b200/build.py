"""Build libllamini_cuda.so in-tree (llamini.cpp_b200/lib/).

CUDA sources are compiled by nvcc for sm_100a only (no other architecture, no
PTX fallback); host C++ by g++ against the CUDA runtime headers. The CUDA
runtime is linked statically, so the library loads on a machine without a GPU
(calls then fail with "no usable CUDA device").
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
LIB = os.path.join(HERE, "lib")
OBJ = os.path.join(HERE, "_build")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INC = ["-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
                     "--expt-relaxed-constexpr"] + INC
CXX_FLAGS = ["-O2", "-fPIC", "-std=c++17", "-Wall", "-I" + os.path.join(CUDA, "include")] + INC


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: %s\n%s%s" % (" ".join(cmd), r.stdout, r.stderr))
    return r.stdout + r.stderr


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_info: bool = False, timeline: bool = False) -> str:
    """Compile every source that changed and relink; returns the .so path.
    timeline = True builds the profiling variant (per-op stamps in the flow
    kernel, flow_timeline.py) into lib_timeline/ instead."""
    lib_dir, obj_dir = (os.path.join(HERE, "lib_timeline"), os.path.join(HERE, "_build_timeline")) if timeline \
        else (LIB, OBJ)
    nvcc_flags = NVCC_FLAGS + (["-DLLAMINI_FLOW_TIMELINE"] if timeline else [])
    os.makedirs(lib_dir, exist_ok=True)
    os.makedirs(obj_dir, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    jobs = []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp"))):
        obj = os.path.join(obj_dir, os.path.basename(src) + ".o")
        if src.endswith(".cu"):
            flags = nvcc_flags + (["-Xptxas", "-v"] if ptxas_info else [])
            cmd = [NVCC] + flags + ["-c", src, "-o", obj]
        else:
            cmd = ["g++"] + CXX_FLAGS + ["-c", src, "-o", obj]
        jobs.append((src, obj, cmd))
    todo = [j for j in jobs if ptxas_info or _stale(j[1], [j[0]] + headers)]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for (src, _, _), out in zip(todo, ex.map(lambda j: _run(j[2]), todo)):
            if verbose and out.strip():
                print("==", os.path.basename(src), "\n" + out)
    so = os.path.join(lib_dir, "libllamini_cuda.so")
    objs = [j[1] for j in jobs]
    if todo or _stale(so, objs):
        _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", so] + objs + ["-lpthread", "-ldl", "-lrt"])
    return so


if __name__ == "__main__":
    print(build(verbose=True, ptxas_info="--ptxas" in sys.argv))
