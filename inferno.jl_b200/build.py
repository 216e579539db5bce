"""Build libinferno_b200.so in-tree with nvcc for sm_100a.

    python inferno.jl_b200/build.py          # or __graft_entry__.build()

The shared library has a C ABI only (include/inferno_b200.h); no torch
extension is involved, so the same .so is what Julia would `ccall`.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libinferno_b200.so")
SOURCES = ["api.cu", "quant.cu", "qgemv.cu", "qmma.cu", "accept.cu", "model.cu", "engine.cu", "comm.cpp", "encode.cpp"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--shared", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-ldl",
    "-Xptxas", "-warn-spills",
    "-I", os.path.join(ROOT, "include"),
]


def sources():
    return [os.path.join(CSRC, s) for s in SOURCES]


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(ROOT, "include", "inferno_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False):
    if not force and not needs_build():
        return LIB
    cmd = [NVCC] + FLAGS + sources() + ["-o", LIB + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libinferno_b200.so")
    if verbose:
        sys.stderr.write(r.stdout + r.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
