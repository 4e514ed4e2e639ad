"""Builds the sm_100a shared library of the MoE hot path in-tree.

    python burn-extended_b200/build.py        # -> burn-extended_b200/mxmoe/libmxmoe.so

Cross-compiles with nvcc (no GPU needed).  The library links the shared CUDA
runtime so that it shares one runtime instance with PyTorch in the same
process.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "mxmoe", "libmxmoe.so")
SOURCES = ["api.cu", "kernels.cu", "dqgemv.cu", "attention.cu", "gemm_tc.cu", "modelbin.cpp", "safetensors.cpp"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-cudart", "shared",
]


def build(verbose: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    deps.append(os.path.join(HERE, "..", "include", "mxmoe.h"))
    if os.path.exists(OUT) and all(os.path.getmtime(OUT) >= os.path.getmtime(d) for d in deps):
        return OUT
    objs = []
    os.makedirs(os.path.join(HERE, "_build"), exist_ok=True)
    for s in srcs:
        o = os.path.join(HERE, "_build", os.path.basename(s) + ".o")
        cmd = [NVCC, *FLAGS, "-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(o)
    cmd = [NVCC, *FLAGS, "-shared", *objs, "-lcublas", "-o", OUT]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
