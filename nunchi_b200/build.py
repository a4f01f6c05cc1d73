"""Build the engine library in-tree: nunchi_b200/libimi_cuda.so (sm_100a kernels + C++ host + C-ABI).

    python -m nunchi_b200.build

nvcc cross-compiles sm_100a without a GPU. Device code is built with --fmad=false so no float multiply-add is
contracted behind the source's back (the kernels spell every fused operation out); host code with -ffp-contract=off
for the same reason (the rotary tables must round exactly as imi's step does).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libimi_cuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
HOST = "-O3,-fPIC,-ffp-contract=off,-fno-math-errno"
SOURCES = ["kernels.cu", "engine.cpp", "gguf_file.cpp", "rope_host.cpp"]


def _stale() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(SRC, f) for f in os.listdir(SRC)] + [os.path.join(HERE, "..", "include", "imi_cuda.h")]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return OUT
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for s in SOURCES:
        o = os.path.join(objdir, os.path.splitext(s)[0] + ".o")
        cmd = [NVCC, "-c", os.path.join(SRC, s), "-o", o, "-std=c++17", "-O3", "-lineinfo", "--fmad=false",
               "-Xcompiler", HOST, *ARCH]
        if s.endswith(".cpp"):
            cmd[1:1] = ["-x", "cu"] if s == "engine.cpp" else []
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(o)
    tmp = OUT + f".tmp{os.getpid()}"
    subprocess.run([NVCC, "-shared", "-o", tmp, *objs, *ARCH, "-lcudart"], check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
