"""Build libllmx.so (CUDA kernels for sm_100a + C++ host runtime + C ABI).

Usage: python llm-accel_b200/build.py [--force] [--timeline]
The shared library is written next to this file so that it travels with the
source tree; nothing is installed into site-packages.  --timeline builds the
measurement variant libllmx_timeline.so instead (-DLLMX_TIMELINE: every launch
of the path stamps its first CTA start and last warp exit with %globaltimer,
read back through llmx_timeline_*; see csrc/timeline.cuh), in its own object
directory; llmx.py loads it when LLMX_TIMELINE=1.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libllmx.so")
ROOT = os.path.dirname(HERE)

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-ffp-contract=off",
          "-I", os.path.join(ROOT, "include"), "-I", CSRC]
SOURCES = ["kernels.cu", "gemv.cu", "attention.cu", "mma_proj.cu", "lm_head.cu", "feature.cu", "runtime.cu", "host_model.cpp",
           "shape.cpp"]


def _nccl():
    """Use the NCCL that torch ships (one libnccl.so.2 per process: the bench and
    tests load torch.distributed next to this library); else the system NCCL."""
    try:
        import nvidia.nccl as n
        base = list(n.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(lib, "libnccl.so.2")):
            return ["-I", inc], ["-L", lib, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + lib]
    except ImportError:
        pass
    return [], ["-lnccl"]


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(ROOT, "include", "llmx.h"))
    return hs


def _compile(src, force, build_dir, defines):
    path = os.path.join(CSRC, src)
    obj = os.path.join(build_dir, src + ".o")
    if not force and not _newer(obj, [path] + _headers()):
        return obj
    cmd = [NVCC, *ARCH, *COMMON, *defines, *_nccl()[0], "-c", path, "-o", obj]
    subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, timeline: bool = False) -> str:
    build_dir = BUILD + "_timeline" if timeline else BUILD
    lib = os.path.join(HERE, "libllmx_timeline.so") if timeline else LIB
    defines = ["-DLLMX_TIMELINE"] if timeline else []
    os.makedirs(build_dir, exist_ok=True)
    with cf.ThreadPoolExecutor(len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, build_dir, defines), SOURCES))
    if force or _newer(lib, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", lib, *objs, *_nccl()[1], "-lpthread"]
        subprocess.run(cmd, check=True)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, timeline="--timeline" in sys.argv))
