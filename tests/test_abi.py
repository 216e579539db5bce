"""CPU checks of the C-ABI library: it loads, exports every symbol declared
in include/inferno_b200.h, and rejects bad arguments without touching a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "inferno_b200.h")
LIB = os.path.join(ROOT, "inferno.jl_b200", "libinferno_b200.so")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"\b([a-z_0-9]+)\s*\(", src)
    skip = {"defined", "sizeof", "push"}
    return sorted({n for n in names if n not in skip})


def test_library_exports_every_declared_symbol(pkg):
    pkg.load()
    lib = ctypes.CDLL(LIB)
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"missing export {n}"
    # and the python binding declares each of them
    assert set(names) == set(pkg._lib.SIGNATURES)


def test_exports_are_only_the_abi():
    """-fvisibility=hidden: nothing but the C ABI leaks out of the .so"""
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == set(declared_functions())


def test_version_and_errors_without_gpu(pkg):
    L = pkg.load()
    assert L.ifr_version() >= 100
    h = ctypes.c_void_p()
    assert L.ifr_ctx_create(0, None) == pkg._lib.IFR_ERR_ARG
    assert b"NULL" in L.ifr_last_error()
    # NULL context / tensor arguments are rejected before any CUDA call
    assert L.ifr_qgemm(None, None, None, 1, None) == pkg._lib.IFR_ERR_ARG
    assert L.ifr_sync(None) == pkg._lib.IFR_ERR_ARG
    assert L.ifr_tensor_free(None) == 0
    assert L.ifr_ctx_destroy(None) == 0
    # the step in parts: NULL states and arguments fail before any device work
    assert L.ifr_draft_mtp(None, 4, None) == pkg._lib.IFR_ERR_ARG
    assert L.ifr_verify_step(None, 4, None, None) == pkg._lib.IFR_ERR_ARG
    assert L.ifr_rollback(None, None, None) == pkg._lib.IFR_ERR_ARG
    assert L.ifr_sample(None, None, 1, 4, ctypes.c_float(1.0), 0, ctypes.c_float(1.0), ctypes.c_float(0.0),
                        None, None) == pkg._lib.IFR_ERR_ARG
    del h


def test_quantized_kernels_kill_switch(pkg, monkeypatch):
    import importlib
    qk = importlib.import_module("inferno_b200.quantized_kernels")
    monkeypatch.setenv("INFERNO_NO_QUANT_KERNELS", "1")
    qk._init()
    assert not qk.quant_kernels_available()
    with pytest.raises(RuntimeError, match="not available"):
        qk.q4_k_gemv_(np.zeros(1, np.float32), np.zeros(144, np.uint8), np.zeros(256, np.float32), 256, 1)
    monkeypatch.setenv("INFERNO_NO_QUANT_KERNELS", "0")
    qk._init()
    assert qk.quant_kernels_available()


def test_row_bytes(pkg):
    assert pkg.row_bytes(pkg.TYPE_Q4_K, 4096) == 16 * 144
    assert pkg.row_bytes(pkg.TYPE_Q6_K, 1024) == 4 * 210
    assert pkg.row_bytes(pkg.TYPE_Q8_0, 1152) == 36 * 34
    with pytest.raises(ValueError):
        pkg.row_bytes(pkg.TYPE_Q4_K, 1000)


def test_accept_rejects_too_many_rows_without_gpu(pkg):
    """batch * (2 gamma + 1) logits rows above 65535 (the statistics kernel's
    grid rows) are IFR_ERR_ARG in both acceptance entry points, checked
    before the context is used (a dummy context pointer is never touched)"""
    L = pkg.load()
    dummy = ctypes.create_string_buffer(4096)
    p = ctypes.cast(dummy, ctypes.c_void_p)
    for fn in ("ifr_accept", "ifr_accept_noalloc"):
        # 8000 x 9 rows at a tiny vocabulary: small scratch, too many rows
        rc = getattr(L, fn)(p, p, p, None, p, 8000, 4, 16, ctypes.c_float(1.0), p, p, None)
        assert rc == pkg._lib.IFR_ERR_ARG, fn
        assert b"rows exceed 65535" in L.ifr_last_error(), fn
