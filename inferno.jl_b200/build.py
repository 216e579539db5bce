"""Build libinferno_b200.so in-tree with nvcc for sm_100a.

    python inferno.jl_b200/build.py          # or __graft_entry__.build()

The shared library has a C ABI only (include/inferno_b200.h); no torch
extension is involved, so the same .so is what Julia would `ccall`.
Each source compiles to its own object under _build/ (in parallel, and only
when the source or a header is newer than its object); the objects are then
linked into the library.
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libinferno_b200.so")
SOURCES = ["api.cu", "quant.cu", "qgemv.cu", "qgemv_q4k.cu", "qgemv_q5k.cu", "qgemv_q6k.cu", "qgemv_q80.cu",
           "qmma.cu", "accept.cu", "model.cu", "engine.cu", "comm.cpp", "encode.cpp"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
    "-I", os.path.join(ROOT, "include"),
]
LDFLAGS = ARCH + ["--shared", "-Xcompiler", "-fPIC", "-ldl"]


def sources():
    return [os.path.join(CSRC, s) for s in SOURCES]


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(ROOT, "include", "inferno_b200.h")]


def obj_of(src):
    return os.path.join(OBJ, os.path.basename(src) + ".o")


def stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def needs_build():
    hs = headers()
    return stale(LIB, sources() + hs) or any(stale(obj_of(s), [s] + hs) for s in sources())


def _compile(src, verbose):
    cmd = [NVCC] + CFLAGS + (["-Xptxas=-v"] if verbose else []) + ["-c", src, "-o", obj_of(src) + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode == 0:
        os.replace(obj_of(src) + ".tmp", obj_of(src))
    return src, r


def build(force=False, verbose=False):
    if not force and not needs_build():
        return LIB
    os.makedirs(OBJ, exist_ok=True)
    hs = headers()
    todo = [s for s in sources() if force or stale(obj_of(s), [s] + hs)]
    failed = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 4))) as ex:
        for src, r in ex.map(lambda s: _compile(s, verbose), todo):
            if verbose or r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                failed.append(os.path.basename(src))
    if failed:
        raise RuntimeError("nvcc failed building libinferno_b200.so: " + ", ".join(failed))
    cmd = [NVCC] + LDFLAGS + [obj_of(s) for s in sources()] + ["-o", LIB + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed linking libinferno_b200.so")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
