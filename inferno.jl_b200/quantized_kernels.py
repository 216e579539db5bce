"""Mirror of the reference's src/QuantizedKernels.jl over libinferno_b200.

Same entry points, argument meaning and error behaviour as the Julia module
(`q4_k_gemv!` is `q4_k_gemv_` here): `out = W * x` for one f32 column, with W
the raw GGUF block bytes of an (outer_dim x inner_dim) matrix.  The reference
binds src/kernels/libquant_kernels.so (QuantizedKernels.jl:22); this module
binds the same C symbols exported by libinferno_b200.so, which run on the GPU.

Arithmetic: like the reference's kernels, these symbols round the
activation column to Q8_K first (d = amax/127, roundf; quantize_row_q8_K,
quant_kernels.c:166-194) and form exact int32 sub-block sums (on the GPU's
integer tensor cores), so results match the reference C kernel up to f32
summation order.  Differences, on purpose: there is no Q8_K scratch pool
(QuantizedKernels.jl:60-72), because the quantized column never leaves the
GPU; and every call copies the whole weight matrix to the device (these are
host-pointer compatibility shims - a model should upload its weights once
through the native ifr_* API instead).
"""
import os

import numpy as np

from . import _lib

_force_disabled = False


def _init():
    # QuantizedKernels.jl:26-32: kill switch
    global _force_disabled
    v = os.environ.get("INFERNO_NO_QUANT_KERNELS")
    _force_disabled = v is not None and v != "0"


_init()


def quant_kernels_available():
    """QuantizedKernels.jl:51: library present and not disabled."""
    if _force_disabled:
        return False
    try:
        _lib.load()
        return True
    except OSError:
        return False


def _require():
    if not quant_kernels_available():
        # QuantizedKernels.jl:86 raises error("Quantized C kernel not available")
        raise RuntimeError("Quantized C kernel not available")
    return _lib.load()


def _call(sym, out, weight_data, x, inner_dim, outer_dim, with_scratch=True):
    L = _require()
    out = np.asarray(out)
    assert out.dtype == np.float32 and out.flags.c_contiguous and out.size >= outer_dim
    w = np.ascontiguousarray(weight_data, dtype=np.uint8)
    xv = np.ascontiguousarray(x, dtype=np.float32)
    if inner_dim % (32 if sym == "q8_0_gemv" else 256):
        # QuantizedKernels.jl:64 asserts inner_dim % 256 == 0 for the K-quants
        raise AssertionError(f"inner_dim={inner_dim} not a multiple of the block size")
    fn = getattr(L, sym)
    args = [w.ctypes.data, xv.ctypes.data, out.ctypes.data]
    if with_scratch:
        args.append(None)
    fn(*args, int(inner_dim), int(outer_dim))
    if np.isnan(out[:outer_dim]).all() and outer_dim > 0:
        raise RuntimeError(L.ifr_last_error().decode())
    return out


def q4_k_gemv_(out, weight_data, x, inner_dim, outer_dim):
    """QuantizedKernels.jl:84-96"""
    return _call("q4_k_gemv", out, weight_data, x, inner_dim, outer_dim)


def q5_k_gemv_(out, weight_data, x, inner_dim, outer_dim):
    """QuantizedKernels.jl:103-115"""
    return _call("q5_k_gemv", out, weight_data, x, inner_dim, outer_dim)


def q6_k_gemv_(out, weight_data, x, inner_dim, outer_dim):
    """QuantizedKernels.jl:122-134"""
    return _call("q6_k_gemv", out, weight_data, x, inner_dim, outer_dim)


def q8_0_gemv_(out, weight_data, x, inner_dim, outer_dim):
    """QuantizedKernels.jl:141-149"""
    return _call("q8_0_gemv", out, weight_data, x, inner_dim, outer_dim, with_scratch=False)
