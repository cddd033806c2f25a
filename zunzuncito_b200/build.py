"""Builds libzz_cuda.so in-tree with nvcc for sm_100a (no JIT cache, so the built
library travels with the source tree). Usage: python zunzuncito_b200/build.py [--force]
It imports nothing from the package, so it can run before the library exists."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libzz_cuda.so")
SOURCES = ["zz_capi.cu", "zz_quant.cu", "zz_gemv.cu", "zz_moe.cu", "zz_moe_i8.cu", "zz_moe_h3.cu", "zz_moe_dec.cu", "zz_ep.cu", "zz_f32act.cu", "zz_route.cu", "zz_loader.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC,-O3", "-Xptxas", "-v" if os.environ.get("ZZ_PTXAS_V") else "-O3",
         "-I" + os.path.join(ROOT, "include")] + os.environ.get("ZZ_NVCC_EXTRA", "").split()


def build(force=False, verbose=False):
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")]
    deps.append(os.path.join(ROOT, "include", "zz_gpu.h"))
    if not force and os.path.exists(LIB):
        t = os.path.getmtime(LIB)
        if all(os.path.getmtime(d) <= t for d in deps):
            return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for s in srcs:
        o = os.path.join(objdir, os.path.basename(s) + ".o")
        cmd = [NVCC, *FLAGS, "-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(o)
    # -z defs: an unresolved symbol is a build error, not a load-time surprise
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xlinker", "-z,defs", "-o", LIB, *objs]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
