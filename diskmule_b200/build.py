"""Build the sm_100a shared library `diskmule_b200/libdiskmule_cuda.so` with nvcc.

The library is the C-ABI boundary declared in include/diskmule_cuda.h. It links
the CUDA runtime statically, so loading it needs only the driver (and loads
without a GPU: every entry point then returns DM_ERR_NO_DEVICE).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libdiskmule_cuda.so")
BUILD = os.path.join(HERE, "_build")

SOURCES = ["dm_kernels.cu", "dm_gemv.cu", "dm_tc.cu", "dm_api.cu", "dm_cache.cu", "dm_stack.cu", "dm_synth.cu", "dm_ep.cu", "dm_gguf.cu", "dm_gemma.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"),
                 shutil.which("nvcc") or ""):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _host_compiler() -> list[str]:
    gxx = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else (shutil.which("g++") or "")
    return ["-ccbin", gxx] if gxx else []


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers += [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]
    common = [nvcc, *ARCH, *_host_compiler(), "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "-Xptxas", "-warn-spills", "--expt-relaxed-constexpr",
              "-DDM_BUILDING_LIBRARY", "-Xcompiler", "-fopenmp", "-Xcompiler", "-ffp-contract=off", "-I", os.path.join(ROOT, "include")]
    objects = []
    for src in SOURCES:
        path = os.path.join(CSRC, src)
        obj = os.path.join(BUILD, src + ".o")
        objects.append(obj)
        if force or _stale(obj, [path, *headers]):
            cmd = [*common, "-c", path, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objects):
        cmd = [nvcc, *ARCH, *_host_compiler(), "-shared", "-cudart", "static", "-o", LIB,
               *objects, "-Xcompiler", "-fopenmp", "-lgomp", "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
