"""ctypes bindings to the CPU oracle (liboracle.so) and to the reference's own
native GEMV kernels compiled from source (_ref/libquant_ref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py, never by the shipped library.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libquant_ref.so")

F32, F16, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 8, 12, 13, 14
TYPE_NAMES = {Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", Q8_0: "Q8_0", F32: "F32", F16: "F16"}
BLOCK = {Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210), Q8_0: (32, 34)}

_lib = None
_ref = None

_fp = ctypes.POINTER(ctypes.c_float)
_dp = ctypes.POINTER(ctypes.c_double)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i32p = ctypes.POINTER(ctypes.c_int32)


def build():
    """Compile liboracle.so (and _ref/ when the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        i64 = ctypes.c_int64
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_f32_to_f16.restype = ctypes.c_uint16
        L.or_f32_to_f16.argtypes = [ctypes.c_float]
        L.or_row_bytes.restype = i64
        L.or_row_bytes.argtypes = [ctypes.c_int, i64]
        L.or_quantize.argtypes = [ctypes.c_int, _fp, i64, i64, _u8p]
        L.or_dequantize.argtypes = [ctypes.c_int, _u8p, i64, _fp]
        L.or_gemm_f64.argtypes = [ctypes.c_int, _u8p, i64, i64, _fp, ctypes.c_int, _dp]
        L.or_gemm_f32.argtypes = [ctypes.c_int, _u8p, i64, i64, _fp, ctypes.c_int, _fp]
        L.or_exp.restype = ctypes.c_float
        L.or_exp.argtypes = [ctypes.c_float]
        L.or_sample_from_probs.argtypes = [_fp, ctypes.c_int, ctypes.c_float]
        L.or_accept.argtypes = [_fp, _fp, _i32p, _fp, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, ctypes.c_float, _i32p, _i32p, _i32p]
        L.or_accept_greedy.argtypes = [_fp, _i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       _i32p, _i32p]
        L.or_argmax.argtypes = [_fp, ctypes.c_int]
        _lib = L
    return _lib


def ref_available():
    return os.path.exists(REF_PATH)


def ref():
    """The reference's quant_kernels.c, built by `make ref`."""
    global _ref
    if _ref is None:
        R = ctypes.CDLL(REF_PATH)
        for n in ("q4_k_gemv", "q5_k_gemv", "q6_k_gemv"):
            getattr(R, n).argtypes = [_u8p, _fp, _fp, _u8p, ctypes.c_int, ctypes.c_int]
            getattr(R, n).restype = None
        R.q8_0_gemv.argtypes = [_u8p, _fp, _fp, ctypes.c_int, ctypes.c_int]
        R.q8_0_gemv.restype = None
        _ref = R
    return _ref


def _p(a, t):
    return a.ctypes.data_as(t)


def row_bytes(qtype, cols):
    return int(lib().or_row_bytes(qtype, cols))


def quantize(qtype, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    rb = row_bytes(qtype, cols)
    assert rb > 0, "cols not a multiple of the block size"
    out = np.empty(rows * rb, dtype=np.uint8)
    assert lib().or_quantize(qtype, _p(x, _fp), rows, cols, _p(out, _u8p)) == 0
    return out


def dequantize(qtype, blocks, n):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    assert lib().or_dequantize(qtype, _p(blocks, _u8p), n, _p(out, _fp)) == 0
    return out


def gemm_f64(qtype, W, rows, cols, X):
    X = np.ascontiguousarray(X, dtype=np.float32).reshape(-1, cols)
    Y = np.empty((X.shape[0], rows), dtype=np.float64)
    assert lib().or_gemm_f64(qtype, _p(np.ascontiguousarray(W), _u8p), rows, cols,
                             _p(X, _fp), X.shape[0], _p(Y, _dp)) == 0
    return Y


def gemm_f32(qtype, W, rows, cols, X):
    X = np.ascontiguousarray(X, dtype=np.float32).reshape(-1, cols)
    Y = np.empty((X.shape[0], rows), dtype=np.float32)
    assert lib().or_gemm_f32(qtype, _p(np.ascontiguousarray(W), _u8p), rows, cols,
                             _p(X, _fp), X.shape[0], _p(Y, _fp)) == 0
    return Y


def ref_gemv(qtype, W, rows, cols, x):
    """One column through the reference's own C kernel (Q8_K activations)."""
    R = ref()
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(rows, dtype=np.float32)
    W = np.ascontiguousarray(W)
    if qtype == Q8_0:
        R.q8_0_gemv(_p(W, _u8p), _p(x, _fp), _p(out, _fp), cols, rows)
    else:
        scratch = np.empty(cols // 256 * 292 + 64, dtype=np.uint8)
        fn = {Q4_K: R.q4_k_gemv, Q5_K: R.q5_k_gemv, Q6_K: R.q6_k_gemv}[qtype]
        fn(_p(W, _u8p), _p(x, _fp), _p(out, _fp), _p(scratch, _u8p), cols, rows)
    return out


def exp(x):
    return float(lib().or_exp(float(x)))


def sample_from_probs(probs, r):
    p = np.ascontiguousarray(probs, dtype=np.float32)
    return int(lib().or_sample_from_probs(_p(p, _fp), len(p), float(r)))


def accept(target, draft, uniforms, temperature, draft_tokens=None):
    target = np.ascontiguousarray(target, dtype=np.float32)
    draft = np.ascontiguousarray(draft, dtype=np.float32)
    uniforms = np.ascontiguousarray(uniforms, dtype=np.float32)
    B, G1, V = target.shape
    G = G1 - 1
    acc = np.empty(B, dtype=np.int32)
    out = np.empty((B, G + 1), dtype=np.int32)
    dout = np.empty((B, G), dtype=np.int32)
    dt = None
    if draft_tokens is not None:
        dt = np.ascontiguousarray(draft_tokens, dtype=np.int32)
    rc = lib().or_accept(_p(target, _fp), _p(draft, _fp),
                         _p(dt, _i32p) if dt is not None else None,
                         _p(uniforms, _fp), B, G, V, float(temperature),
                         _p(acc, _i32p), _p(out, _i32p), _p(dout, _i32p))
    assert rc == 0
    return acc, out, dout


def accept_greedy(target, draft_tokens):
    target = np.ascontiguousarray(target, dtype=np.float32)
    B, G1, V = target.shape
    dt = np.ascontiguousarray(draft_tokens, dtype=np.int32).reshape(B, G1 - 1)
    acc = np.empty(B, dtype=np.int32)
    out = np.empty((B, G1), dtype=np.int32)
    assert lib().or_accept_greedy(_p(target, _fp), _p(dt, _i32p), B, G1 - 1, V,
                                  _p(acc, _i32p), _p(out, _i32p)) == 0
    return acc, out


def norm_rel(a, b):
    """||a-b|| / ||b|| per leading row (the GEMV/logits parity metric)."""
    a = np.asarray(a, dtype=np.float64).reshape(-1, np.shape(b)[-1])
    b = np.asarray(b, dtype=np.float64).reshape(a.shape)
    den = np.linalg.norm(b, axis=1)
    den[den == 0] = 1.0
    return np.linalg.norm(a - b, axis=1) / den
