"""Builds the B200 matmul library in-tree.

    python llm-engine_b200/build.py          # incremental
    python llm-engine_b200/build.py --force  # rebuild everything

Outputs (git-ignored, they travel with the source tree):
    llm-engine_b200/lib/libllme_b200.so      kernels + the C ABI (include/llme_b200.h)
    llm-engine_b200/lib/libllme_b200_cxx.so  the drop-in C++ API (include/cuda_matmul.h)

Every CUDA source is compiled for sm_100a only (-gencode arch=compute_100a,code=sm_100a);
the CUDA runtime is linked statically so the library does not depend on which libcudart
a host process (e.g. PyTorch's) has already loaded.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "lib")

CUDA_SOURCES = ["capi.cu", "gemv.cu", "gemm_simt.cu", "gemm_tc.cu", "gemm_q8_tc.cu", "gemm_q8_skinny.cu", "gemm_f32_skinny.cu", "quant.cu", "decode_ops.cu", "attention.cu", "comm.cu", "model.cu"]
CXX_SHIM = "cuda_matmul.cpp"
LIB_NAME = "libllme_b200.so"
CXX_LIB_NAME = "libllme_b200_cxx.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-Wall", "-I" + INCLUDE, "-I" + CSRC,
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the B200 library cannot be built")


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    """Compiles and links; returns the path of libllme_b200.so."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    headers = _headers()
    nv = nvcc()
    objs, jobs = [], []
    for src in CUDA_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src + ".o")
        objs.append(o)
        if force or ptxas_info or _stale(o, [s] + headers):
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            jobs.append([nv] + NVCC_FLAGS + extra + ["-c", s, "-o", o])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for out in ex.map(lambda c: _run(c, verbose), jobs):
                if ptxas_info and out:
                    print(out)
    lib = os.path.join(LIB, LIB_NAME)
    if force or _stale(lib, objs):
        _run([nv] + ARCH + ["-shared", "-o", lib] + objs + ["-ldl"], verbose)
    cxx = os.path.join(LIB, CXX_LIB_NAME)
    shim = os.path.join(CSRC, CXX_SHIM)
    if force or _stale(cxx, [shim, lib] + headers):
        gxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
        _run([gxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-Wextra",
              "-I" + INCLUDE, "-I" + os.path.join(INCLUDE, "tensor"), shim, "-o", cxx,
              "-L" + LIB, "-lllme_b200", "-Wl,-rpath,$ORIGIN"], verbose)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))
    sys.exit(0)
