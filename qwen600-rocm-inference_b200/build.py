"""Build the engine's shared library in-tree: lib/libqwen_b200.so (sm_100a).

    python qwen600-rocm-inference_b200/build.py [--force]

nvcc compiles the CUDA translation unit for sm_100a only
(-gencode arch=compute_100a,code=sm_100a); the host-only C++ files go through
nvcc's host compiler with the same flags.  The CUDA runtime is linked
statically, so the library needs only the driver at run time.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "lib")
OUT = os.path.join(LIB, "libqwen_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

CUDA_SOURCES = ["engine.cu"]
HOST_SOURCES = ["model_format.cpp", "host_sampler.cpp", "tokenizer.cpp"]
HEADERS = ["decode_kernel.cuh", "attention_tc5.cuh", "gemv_kernel.cuh", "gemm_tc.cuh", "prefill_kernels.cuh", "ptx.cuh", "model_format.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fopenmp", "-I", os.path.join(HERE, "..", "include")]


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force=False, verbose_ptxas=False):
    os.makedirs(LIB, exist_ok=True)
    objdir = os.path.join(LIB, "obj")
    os.makedirs(objdir, exist_ok=True)
    deps = [os.path.join(CSRC, f) for f in CUDA_SOURCES + HOST_SOURCES + HEADERS]
    deps += [os.path.join(HERE, "host", "config.h"), os.path.join(HERE, "..", "include", "qwen_b200.h"), __file__]
    if not force and not _stale(OUT, deps):
        return OUT
    objs = []
    for src in CUDA_SOURCES:
        obj = os.path.join(objdir, src + ".o")
        extra = ["-Xptxas", "-v"] if verbose_ptxas else []
        _run([NVCC, *ARCH, "-lineinfo", *COMMON, *extra, "-c", os.path.join(CSRC, src), "-o", obj])
        objs.append(obj)
    for src in HOST_SOURCES:
        obj = os.path.join(objdir, src + ".o")
        _run([NVCC, *COMMON, "-Wno-deprecated-gpu-targets", "-x", "c++", "-c", os.path.join(CSRC, src), "-o", obj])
        objs.append(obj)
    tmp = OUT + ".tmp"
    _run([NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lgomp"])
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="--ptxas" in sys.argv)
