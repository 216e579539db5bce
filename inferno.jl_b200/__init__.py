"""inferno_b200: host side of the B200 speculative-decoding verify path.

The package directory is ``inferno.jl_b200/``; load it with
``__graft_entry__.load_package()`` (it registers the module as
``inferno_b200``).  Everything here is a thin layer over the C ABI of
libinferno_b200.so; torch is used only to own device memory and streams.

Modules
  _lib                ctypes binding of every C symbol (include/inferno_b200.h)
  quantized_kernels   mirror of the reference's src/QuantizedKernels.jl
                      (q4_k_gemv! ... q8_0_gemv!, kill switch, availability)
  speculative         mirror of src/SpeculativeDecoding.jl acceptance entry points
"""
import ctypes

import numpy as np

from . import _lib
from ._lib import (IfrError, MAX_VERIFY_COLS, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_0,  # noqa: F401
                   check, load)

__all__ = ["Context", "QTensor", "IfrError", "load", "TYPE_Q4_K", "TYPE_Q5_K", "TYPE_Q6_K",
           "TYPE_Q8_0", "row_bytes"]

BLOCK = {TYPE_Q4_K: (256, 144), TYPE_Q5_K: (256, 176), TYPE_Q6_K: (256, 210), TYPE_Q8_0: (32, 34)}


def row_bytes(qtype, cols):
    be, bb = BLOCK[qtype]
    if cols % be:
        raise ValueError(f"cols={cols} is not a multiple of {be}")
    return cols // be * bb


def quantize(qtype, x):
    """f32 rows (numpy [rows, cols]) -> GGUF block bytes, the library's host encoder"""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty(rows * row_bytes(qtype, cols), dtype=np.uint8)
    check(load().ifr_quantize(qtype, x.ctypes.data_as(ctypes.c_void_p), rows, cols,
                              out.ctypes.data_as(ctypes.c_void_p)))
    return out


def _ptr(t):
    """device pointer of a torch tensor (or None)"""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


class QTensor:
    """A device-resident quantized weight matrix (rows x cols) owned by the library."""

    def __init__(self, ctx, handle, qtype, rows, cols):
        self.ctx, self.handle, self.qtype, self.rows, self.cols = ctx, handle, qtype, rows, cols

    def device_bytes(self):
        b = ctypes.c_int64()
        check(load().ifr_tensor_info(self.handle, None, None, None, ctypes.byref(b)))
        return b.value

    def algorithmic_bytes(self):
        return self.rows * row_bytes(self.qtype, self.cols)

    def free(self):
        if self.handle:
            load().ifr_tensor_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Context:
    """One device + one stream.  By default the library launches on torch's
    current stream, so its kernels are ordered with torch work."""

    def __init__(self, device=0, torch_stream=True):
        import torch
        self.torch = torch
        self.device = device
        L = load()
        h = ctypes.c_void_p()
        check(L.ifr_ctx_create(device, ctypes.byref(h)))
        self.handle = h
        if torch_stream:
            with torch.cuda.device(device):
                s = torch.cuda.current_stream().cuda_stream
            check(L.ifr_ctx_set_stream(self.handle, ctypes.c_void_p(s)))

    def close(self):
        if getattr(self, "handle", None):
            load().ifr_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    ACT_EXACT, ACT_Q8K = 0, 1

    def set_activation(self, mode):
        """K-quant GEMV activations: ACT_EXACT (default, exact f32) or ACT_Q8K
        (Q8_K-quantised, the reference's kernels)"""
        check(load().ifr_ctx_set_activation(self.handle, int(mode)))

    def set_dense_min_cols(self, ncols):
        """engine projections of >= ncols columns use the dense tensor-core path"""
        check(load().ifr_ctx_set_dense_min_cols(self.handle, int(ncols)))

    def set_prefill_dense(self, enable=True):
        """let one-request prefill chunks use the dense tensor-core path"""
        check(load().ifr_ctx_set_prefill_dense(self.handle, 1 if enable else 0))

    def set_kv_bf16(self, enable=True):
        """ifr_ctx_set_kv_bf16: split-KV states created afterwards keep bf16
        attention caches (rows rounded to nearest even as they are written)"""
        check(load().ifr_ctx_set_kv_bf16(self.handle, 1 if enable else 0))

    def set_dense_f16_weights(self, enable=True):
        """batched states keep fp16 operand stages of the weights for the dense GEMM"""
        check(load().ifr_ctx_set_dense_f16_weights(self.handle, 1 if enable else 0))

    def prepare_dense(self, W):
        """fp16 operand stages of tensor W for qgemm_dense (same results, no dequant)"""
        check(load().ifr_tensor_prepare_dense(self.handle, W.handle))

    def set_fused_layers(self, enable=True):
        """run a one-request verify's decoder layers as one persistent launch"""
        check(load().ifr_ctx_set_fused_layers(self.handle, 1 if enable else 0))

    def set_stream(self, stream):
        check(load().ifr_ctx_set_stream(self.handle, ctypes.c_void_p(stream.cuda_stream)))

    def reserve_accept(self, batch, gamma, vocab):
        check(load().ifr_ctx_reserve_accept(self.handle, int(batch), int(gamma), int(vocab)))

    def sync(self):
        check(load().ifr_sync(self.handle))

    # --- weights ---------------------------------------------------------
    def upload(self, qtype, blocks, rows, cols):
        """GGUF block bytes (host numpy uint8) -> device QTensor"""
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        if blocks.size != rows * row_bytes(qtype, cols):
            raise ValueError("byte count does not match rows x cols")
        h = ctypes.c_void_p()
        check(load().ifr_weights_upload(self.handle, qtype, blocks.ctypes.data_as(ctypes.c_void_p),
                                        rows, cols, ctypes.byref(h)))
        return QTensor(self, h, qtype, rows, cols)

    def from_device(self, qtype, dev_bytes, rows, cols):
        """GGUF block bytes already on the device (torch uint8 tensor)"""
        h = ctypes.c_void_p()
        check(load().ifr_weights_from_device(self.handle, qtype, _ptr(dev_bytes), rows, cols,
                                             ctypes.byref(h)))
        return QTensor(self, h, qtype, rows, cols)

    # --- compute -----------------------------------------------------------
    def dequant(self, W, out=None):
        torch = self.torch
        if out is None:
            out = torch.empty(W.rows, W.cols, dtype=torch.float32, device=f"cuda:{self.device}")
        check(load().ifr_dequant(self.handle, W.handle, _ptr(out)))
        return out

    def qgemm(self, W, X, out=None):
        """X [ncols, cols] f32 (device) -> Y [ncols, rows]"""
        torch = self.torch
        assert X.dtype == torch.float32 and X.is_contiguous() and X.shape[-1] == W.cols
        n = X.numel() // W.cols
        if out is None:
            out = torch.empty(n, W.rows, dtype=torch.float32, device=X.device)
        check(load().ifr_qgemm(self.handle, W.handle, _ptr(X), n, _ptr(out)))
        return out

    def qgemm_rmsnorm(self, W, X, norm_w, eps, out=None):
        """X [ncols, cols] f32 (device) -> Y [ncols, rows] = W RMSNorm(X; norm_w, eps)"""
        torch = self.torch
        assert X.dtype == torch.float32 and X.is_contiguous() and X.shape[-1] == W.cols
        assert norm_w.dtype == torch.float32 and norm_w.is_contiguous() and norm_w.numel() == W.cols
        n = X.numel() // W.cols
        if out is None:
            out = torch.empty(n, W.rows, dtype=torch.float32, device=X.device)
        check(load().ifr_qgemm_rmsnorm(self.handle, W.handle, _ptr(X), n, _ptr(norm_w), ctypes.c_float(eps),
                                       _ptr(out)))
        return out

    def qgemm_dense(self, W, X, out=None):
        """X [ncols, cols] f32 (device) -> Y [ncols, rows] on the tensor cores
        (fp16 operands, f32 accumulation)"""
        torch = self.torch
        assert X.dtype == torch.float32 and X.is_contiguous() and X.shape[-1] == W.cols
        n = X.numel() // W.cols
        if out is None:
            out = torch.empty(n, W.rows, dtype=torch.float32, device=X.device)
        check(load().ifr_qgemm_dense(self.handle, W.handle, _ptr(X), n, _ptr(out)))
        return out

    def accept(self, target, draft, uniforms, temperature, draft_tokens=None):
        """sampled verification; returns (accept_count, out_tokens, draft_tokens)"""
        torch = self.torch
        B, G1, V = target.shape
        G = G1 - 1
        dev = target.device
        acc = torch.empty(B, dtype=torch.int32, device=dev)
        out = torch.empty(B, G + 1, dtype=torch.int32, device=dev)
        dout = torch.empty(B, G, dtype=torch.int32, device=dev)
        check(load().ifr_accept(self.handle, _ptr(target), _ptr(draft), _ptr(draft_tokens),
                                _ptr(uniforms), B, G, V, float(temperature), _ptr(acc), _ptr(out),
                                _ptr(dout)))
        return acc, out, dout

    def accept_filtered(self, target, draft, uniforms, temperature, top_k=0, top_p=1.0, min_p=0.0):
        """sampled verification on the top-k / top-p / min-p filtered
        distributions; returns (accept_count, out_tokens, draft_tokens)"""
        torch = self.torch
        B, G1, V = target.shape
        G = G1 - 1
        dev = target.device
        acc = torch.empty(B, dtype=torch.int32, device=dev)
        out = torch.empty(B, G + 1, dtype=torch.int32, device=dev)
        dout = torch.empty(B, G, dtype=torch.int32, device=dev)
        check(load().ifr_accept_filtered(self.handle, _ptr(target), _ptr(draft), _ptr(uniforms), B, G, V,
                                         float(temperature), int(top_k), float(top_p), float(min_p), _ptr(acc),
                                         _ptr(out), _ptr(dout)))
        return acc, out, dout

    def sample(self, logits, uniforms, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, out=None):
        """logits [..., vocab] f32 (device), one uniform per row -> int32 tokens
        (0-based; -1 marks a row with NaN or +Inf)"""
        torch = self.torch
        assert logits.dtype == torch.float32 and logits.is_contiguous()
        V = logits.shape[-1]
        rows = logits.numel() // V
        assert uniforms.dtype == torch.float32 and uniforms.is_contiguous() and uniforms.numel() == rows
        if out is None:
            out = torch.empty(rows, dtype=torch.int32, device=logits.device)
        check(load().ifr_sample(self.handle, _ptr(logits), rows, V, ctypes.c_float(temperature), int(top_k),
                                ctypes.c_float(top_p), ctypes.c_float(min_p), _ptr(uniforms), _ptr(out)))
        return out

    def apply_penalties(self, logits, seen, presence=0.0, repetition=1.0):
        """in place on logits [rows, vocab] (device); seen [rows, n] int32 (device)"""
        torch = self.torch
        assert logits.dtype == torch.float32 and logits.is_contiguous()
        assert seen.dtype == torch.int32 and seen.is_contiguous()
        V = logits.shape[-1]
        rows = logits.numel() // V
        n = seen.numel() // max(rows, 1)
        check(load().ifr_apply_penalties(self.handle, _ptr(logits), rows, V, _ptr(seen), n,
                                         ctypes.c_float(presence), ctypes.c_float(repetition)))
        return logits

    def accept_greedy(self, target, draft_tokens):
        torch = self.torch
        B, G1, V = target.shape
        acc = torch.empty(B, dtype=torch.int32, device=target.device)
        out = torch.empty(B, G1, dtype=torch.int32, device=target.device)
        check(load().ifr_accept_greedy(self.handle, _ptr(target), _ptr(draft_tokens), B, G1 - 1, V,
                                       _ptr(acc), _ptr(out)))
        return acc, out
