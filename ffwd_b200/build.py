"""Build the in-tree shared libraries of the B200 backend.

* ``ffwd_b200/lib/libffwd_b200.so`` — CUDA kernels (sm_100a) + host runtime,
  exporting the C ABI of ``include/ffwd_b200.h``.
* ``ffwd_b200/lib/libffwd_b200_api.so`` — the same plus the reference-facing
  public API of ``libffwd/ffwd.h`` (``ffwd_init`` / ``ffwd_open`` /
  ``ffwd_encode_batch`` ...), implemented by ``backend/backend_b200.c``.

nvcc cross-compiles without a GPU; objects go to ``_build/`` (ignored).
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
OBJDIR = os.path.join(ROOT, "_build", "ffwd_b200")
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                  "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]
CU_SRCS = ["gemm.cu", "gemm2.cu", "attention.cu", "rowops.cu", "late.cu", "engine.cu"]
CC_SRCS = ["loader.cc"]

LIB = os.path.join(LIBDIR, "libffwd_b200.so")
API_LIB = os.path.join(LIBDIR, "libffwd_b200_api.so")


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[-1]}")
    return r


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(ROOT, "include", "ffwd_b200.h"))
    jobs = []
    objs = []
    for src in CU_SRCS + CC_SRCS:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJDIR, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            if src.endswith(".cu"):
                cmd = [NVCC] + NVFLAGS + ["-c", s, "-o", o]
            else:
                cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-fvisibility=hidden",
                       "-I/usr/local/cuda/include", "-I" + os.path.join(ROOT, "include"),
                       "-c", s, "-o", o]
            jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        for r in ex.map(_run, jobs):
            if verbose and r.stderr:
                sys.stderr.write(r.stderr)
    if force or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lpthread"])
    api_src = os.path.join(HERE, "backend", "backend_b200.c")
    api_obj = os.path.join(OBJDIR, "backend_b200.o")
    if force or _stale(api_obj, [api_src] + headers):
        _run(["gcc", "-O2", "-std=c11", "-fPIC", "-fvisibility=hidden", "-D_DEFAULT_SOURCE",
              "-I" + os.path.join(ROOT, "include"), "-c", api_src, "-o", api_obj])
    if force or _stale(API_LIB, objs + [api_obj]):
        _run([NVCC] + ARCH + ["-shared", "-o", API_LIB] + objs + [api_obj, "-lpthread"])
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
