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
        L.or_gemm_q8k.argtypes = [ctypes.c_int, _u8p, i64, i64, _fp, ctypes.c_int, _dp]
        L.or_quantize_q8k.argtypes = [_fp, i64, _fp, ctypes.POINTER(ctypes.c_int8)]
        L.or_quantize_q8k.restype = None
        L.or_gemm_f32.argtypes = [ctypes.c_int, _u8p, i64, i64, _fp, ctypes.c_int, _fp]
        L.or_exp.restype = ctypes.c_float
        L.or_exp.argtypes = [ctypes.c_float]
        L.or_sample_from_probs.argtypes = [_fp, ctypes.c_int, ctypes.c_float]
        L.or_accept.argtypes = [_fp, _fp, _i32p, _fp, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, ctypes.c_float, _i32p, _i32p, _i32p]
        L.or_accept_greedy.argtypes = [_fp, _i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       _i32p, _i32p]
        L.or_argmax.argtypes = [_fp, ctypes.c_int]
        L.or_sample_filtered.argtypes = [_fp, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_float,
                                         ctypes.c_float, ctypes.c_float]
        L.or_sample_rows.argtypes = [_fp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                     ctypes.c_float, ctypes.c_float, _fp, _i32p]
        L.or_apply_penalties.argtypes = [_fp, ctypes.c_int, ctypes.c_int, _i32p, ctypes.c_int, ctypes.c_float,
                                         ctypes.c_float]
        L.or_apply_penalties.restype = None
        L.or_accept_filtered.argtypes = [_fp, _fp, _fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                         ctypes.c_int, ctypes.c_float, ctypes.c_float, _i32p, _i32p, _i32p]
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


def gemm_q8k(qtype, W, rows, cols, X):
    """K-quant weights against Q8_K-quantised activations, f64 sums"""
    X = np.ascontiguousarray(X, dtype=np.float32).reshape(-1, cols)
    Y = np.empty((X.shape[0], rows), dtype=np.float64)
    assert lib().or_gemm_q8k(qtype, _p(np.ascontiguousarray(W), _u8p), rows, cols,
                             _p(X, _fp), X.shape[0], _p(Y, _dp)) == 0
    return Y


def gemm_ref(qtype, W, rows, cols, X, act=0):
    """the GPU GEMV's semantics: exact f32 activations (act 0, default), or for
    the K-quants Q8_K activations (act 1, the reference's q4_k_gemv ..
    q6_k_gemv); Q8_0 always exact (the reference's q8_0_gemv)"""
    if qtype == 8 or act == 0:
        return gemm_f64(qtype, W, rows, cols, X)
    return gemm_q8k(qtype, W, rows, cols, X)


def quantize_q8k(x):
    """quantize_row_q8_K restated: (d per 256 block, int8 values)"""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    d = np.empty(len(x) // 256, np.float32)
    q = np.empty(len(x), np.int8)
    lib().or_quantize_q8k(_p(x, _fp), len(x), _p(d, _fp), q.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)))
    return d, q


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


def ref_quantize_q8k(x):
    """quantize_row_q8_K of the reference (oracle/_ref): (d per block, int8),
    or None when oracle/_ref is not built"""
    if not os.path.exists(REF_PATH):
        return None
    R = ref()
    R.quantize_row_q8_K.argtypes = [_fp, _u8p, ctypes.c_int64]
    R.quantize_row_q8_K.restype = None
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    nb = len(x) // 256
    buf = np.empty(nb * 292, np.uint8)  # block_q8_K: f32 d, int8 qs[256], int16 bsums[16]
    R.quantize_row_q8_K(_p(x, _fp), _p(buf, _u8p), len(x))
    blocks = buf.reshape(nb, 292)
    return blocks[:, :4].copy().view(np.float32).ravel(), blocks[:, 4:260].copy().view(np.int8).ravel()


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


def sample(logits, uniforms, temperature=1.0, top_k=0, top_p=1.0, min_p=0.0):
    """filtered sampling per row (CommonOps.jl:196-318): 0-based tokens, -1
    for a row holding NaN or +Inf"""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    V = logits.shape[-1]
    rows = logits.size // V
    u = np.ascontiguousarray(uniforms, dtype=np.float32).reshape(rows)
    out = np.empty(rows, dtype=np.int32)
    lib().or_sample_rows(_p(logits, _fp), rows, V, float(temperature), int(top_k), float(top_p), float(min_p),
                         _p(u, _fp), _p(out, _i32p))
    return out


def accept_filtered(target, draft, uniforms, temperature, top_k=0, top_p=1.0, min_p=0.0):
    """sampled verification on the filtered target and draft distributions:
    (accept counts [B], emitted tokens [B][G+1] (-1 padded), drawn drafts [B][G])"""
    target = np.ascontiguousarray(target, dtype=np.float32)
    draft = np.ascontiguousarray(draft, dtype=np.float32)
    uniforms = np.ascontiguousarray(uniforms, dtype=np.float32)
    B, G1, V = target.shape
    G = G1 - 1
    acc = np.empty(B, dtype=np.int32)
    out = np.empty((B, G + 1), dtype=np.int32)
    dout = np.empty((B, G), dtype=np.int32)
    rc = lib().or_accept_filtered(_p(target, _fp), _p(draft, _fp), _p(uniforms, _fp), B, G, V, float(temperature),
                                  int(top_k), float(top_p), float(min_p), _p(acc, _i32p), _p(out, _i32p),
                                  _p(dout, _i32p))
    assert rc == 0
    return acc, out, dout


def apply_penalties(logits, seen, presence=0.0, repetition=1.0):
    """presence then repetition penalty on each row's distinct seen tokens
    (ModelCPU.jl:1202-1238, CommonOps.jl:63-76); returns a new array"""
    out = np.array(logits, dtype=np.float32, order="C", copy=True)
    V = out.shape[-1]
    rows = out.size // V
    sn = np.ascontiguousarray(seen, dtype=np.int32).reshape(rows, -1)
    lib().or_apply_penalties(_p(out, _fp), rows, V, _p(sn, _i32p), sn.shape[1], float(presence), float(repetition))
    return out


def accept_greedy(target, draft_tokens):
    target = np.ascontiguousarray(target, dtype=np.float32)
    B, G1, V = target.shape
    dt = np.ascontiguousarray(draft_tokens, dtype=np.int32).reshape(B, G1 - 1)
    acc = np.empty(B, dtype=np.int32)
    out = np.empty((B, G1), dtype=np.int32)
    assert lib().or_accept_greedy(_p(target, _fp), _p(dt, _i32p), B, G1 - 1, V,
                                  _p(acc, _i32p), _p(out, _i32p)) == 0
    return acc, out


def _kq_scales(s):
    """6-bit sub-block scales and mins of Q4_K/Q5_K headers (src/Dequant.jl:345-362)"""
    s = s.astype(np.int64)
    sc = np.empty((s.shape[0], 8), np.int64)
    m = np.empty((s.shape[0], 8), np.int64)
    for j in range(4):
        sc[:, j] = s[:, j] & 63
        m[:, j] = s[:, j + 4] & 63
    for j in range(4, 8):
        sc[:, j] = (s[:, j + 4] & 0x0F) | ((s[:, j - 4] >> 6) << 4)
        m[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    return sc, m


def dense_fp16_weights(qtype, blocks, rows, cols):
    """The fp16 weights of the dense tensor-core GEMM (ifr_qgemm_dense), formed
    from the exact integer quants of the GGUF blocks: Q4_K/Q5_K
    fp16(q * fp16(d sc) - fp16(dmin m)), Q6_K fp16((q - 32) fp16(d sc)),
    Q8_0 fp16(q d), each a single rounding of the exact value (f64 here)."""
    be, bb = BLOCK[qtype]
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, bb)
    nb = b.shape[0]
    f16 = lambda a: a.copy().view(np.float16).astype(np.float64)  # noqa: E731
    e = np.arange(be)
    if qtype in (Q4_K, Q5_K):
        d = f16(b[:, 0:2])
        dmin = f16(b[:, 2:4])
        sc, m = _kq_scales(b[:, 4:16])
        qs = b[:, 48:176] if qtype == Q5_K else b[:, 16:144]
        l = e % 32
        q = (qs[:, 32 * (e // 64) + l].astype(np.int64) >> (4 * ((e % 64) >= 32))) & 15
        j = e // 32
        if qtype == Q5_K:
            q = q + 16 * ((b[:, 16 + l].astype(np.int64) >> j) & 1)
        d1 = (d * sc).astype(np.float16).astype(np.float64)[:, j]
        m1 = (dmin * m).astype(np.float16).astype(np.float64)[:, j]
        w = q * d1 - m1
    elif qtype == Q6_K:
        d = f16(b[:, 208:210])
        sc = b[:, 192:208].view(np.int8).astype(np.float64)
        n, qq, l = e // 128, (e % 128) // 32, e % 32
        lo = (b[:, 64 * n + 32 * (qq % 2) + l].astype(np.int64) >> (4 * (qq // 2))) & 15
        hi = (b[:, 128 + 32 * n + l].astype(np.int64) >> (2 * qq)) & 3
        ds = (d * sc).astype(np.float16).astype(np.float64)[:, e // 16]
        w = ((lo | (hi << 4)) - 32) * ds
    else:
        d = f16(b[:, 0:2])
        w = b[:, 2:34].view(np.int8).astype(np.float64) * d
    return w.astype(np.float16).reshape(rows, cols)


def norm_rel(a, b):
    """||a-b|| / ||b|| per leading row (the GEMV/logits parity metric)."""
    a = np.asarray(a, dtype=np.float64).reshape(-1, np.shape(b)[-1])
    b = np.asarray(b, dtype=np.float64).reshape(a.shape)
    den = np.linalg.norm(b, axis=1)
    den[den == 0] = 1.0
    return np.linalg.norm(a - b, axis=1) / den


# ---------------------------------------------------------------- model ----

class _Cfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("hidden", "n_layers", "n_head", "n_kv_head", "head_dim",
                                              "rotary_dim", "ffn", "vocab", "ssm_heads", "ssm_head_dim",
                                              "conv_kernel", "max_ctx")] + [
        ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float)]


_KIND = {"attn_norm.weight": 10, "post_attention_norm.weight": 11, "attn_qkv.weight": 12,
         "attn_gate.weight": 13, "ssm_out.weight": 14, "ssm_conv1d.weight": 15, "ssm_alpha.weight": 16,
         "ssm_beta.weight": 17, "ssm_a": 18, "ssm_dt.bias": 19, "ssm_norm.weight": 20,
         "attn_q.weight": 21, "attn_k.weight": 22, "attn_v.weight": 23, "attn_output.weight": 24,
         "attn_q_norm.weight": 25, "attn_k_norm.weight": 26, "ffn_gate.weight": 27, "ffn_up.weight": 28,
         "ffn_down.weight": 29, "ffn_norm.weight": 30, "post_ffw_norm.weight": 31, "layer_scalar": 32,
         "pli_gate.weight": 40, "pli_proj.weight": 41, "pli_post_norm.weight": 42}
_GLOBAL = {"token_embd.weight": 0, "output_norm.weight": 1, "mtp.fc.weight": 2,
           "mtp.pre_fc_norm_embedding.weight": 3, "mtp.pre_fc_norm_hidden.weight": 4, "mtp.norm.weight": 5,
           "pli_token_embd.weight": 50, "pli_model_proj.weight": 51, "pli_proj_norm.weight": 52}


class _GemmaCfg(ctypes.Structure):
    _fields_ = [("window", ctypes.c_int32), ("sliding_pattern", ctypes.c_int32)] + [
        (n, ctypes.c_float) for n in ("attn_softcap", "final_softcap", "rope_theta_swa", "rope_theta_full",
                                      "partial_rotary_factor", "embed_scale")] + [("pli", ctypes.c_int32)]


def gemma_config(md, hidden):
    """Gemma4 block parameters from GGUF metadata (general.architecture
    "gemma4"; keys as the synthetic models write them)"""
    g = lambda k, dflt: md.get(f"gemma4.{k}", dflt)  # noqa: E731
    return _GemmaCfg(int(g("attention.sliding_window", 512)), int(g("attention.sliding_window_pattern", 6)),
                     float(g("attn_logit_softcapping", 0.0)), float(g("final_logit_softcapping", 0.0)),
                     float(g("rope.freq_base_swa", 10000.0)), float(g("rope.freq_base", 1000000.0)),
                     float(g("rope.partial_rotary_factor", 0.25)),
                     float(np.float32(np.sqrt(np.float64(hidden)))),
                     int(g("embedding_length_per_layer_input", 0)))


def _model_lib():
    L = lib()
    if not hasattr(L, "_model_init"):
        L.or_model_set_gemma.argtypes = [ctypes.c_void_p, ctypes.POINTER(_GemmaCfg)]
        L.or_model_set_gemma.restype = None
        L.or_model_new.restype = ctypes.c_void_p
        L.or_model_new.argtypes = [ctypes.POINTER(_Cfg)]
        L.or_model_free.argtypes = [ctypes.c_void_p]
        L.or_model_set.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                   ctypes.c_int64]
        L.or_model_reset.argtypes = [ctypes.c_void_p]
        L.or_model_set_activation.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.or_model_set_activation.restype = None
        L.or_model_set_kv_bf16.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.or_model_set_kv_bf16.restype = None
        L.or_forward_token.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _fp, _fp]
        L.or_mtp_step.argtypes = [ctypes.c_void_p, ctypes.c_int, _fp, ctypes.c_int, _fp, _fp]
        L.or_snapshot_take.restype = ctypes.c_void_p
        L.or_snapshot_take.argtypes = [ctypes.c_void_p]
        L.or_snapshot_restore.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.or_snapshot_free.argtypes = [ctypes.c_void_p]
        L._model_init = True
    return L


class OracleModel:
    """forward_cpu! restated in C (model.c), loaded from a GGUF file read with
    the package's GGUF reader."""

    def __init__(self, gguf_file, max_ctx):
        f = gguf_file
        md = f.metadata
        arch = md.get("general.architecture", "qwen")
        g = lambda k, dflt: md.get(f"{arch}.{k}", md.get(k, dflt))  # noqa: E731
        emb = f.tensors["token_embd.weight"]
        self.hidden, self.vocab = int(emb.dims[0]), int(emb.dims[1])
        hd = int(g("attention.key_length", 256))
        ssm_heads, ssm_hd = 0, 0
        for i in range(int(g("block_count", 24))):
            if f"blk.{i}.ssm_a" in f.tensors:
                ssm_heads = f.tensors[f"blk.{i}.ssm_a"].n_elements
                ssm_hd = int(f.tensors[f"blk.{i}.attn_gate.weight"].dims[1]) // ssm_heads
                break
        self.cfg = _Cfg(self.hidden, int(g("block_count", 24)), int(g("attention.head_count", 8)),
                        int(g("attention.head_count_kv", 2)), hd,
                        int(round(hd * float(g("rope.partial_rotary_factor", 0.25)))),
                        int(g("feed_forward_length", 3584)), self.vocab, ssm_heads, ssm_hd,
                        int(g("ssm.conv_kernel", 4)), int(max_ctx),
                        float(g("rope.freq_base", 1e7)), float(g("attention.layer_norm_rms_epsilon", 1e-6)))
        L = _model_lib()
        self.L = L
        self.h = L.or_model_new(ctypes.byref(self.cfg))
        for name, ti in f.tensors.items():
            if name in _GLOBAL:
                layer, kind = -1, _GLOBAL[name]
            elif name.startswith("blk."):
                _, idx, rest = name.split(".", 2)
                layer, kind = int(idx), _KIND[rest]
            elif name.startswith("mtp.blk.0."):
                layer, kind = -2, _KIND[name[len("mtp.blk.0."):]]
            else:
                continue
            raw = np.ascontiguousarray(f.raw(name))
            assert L.or_model_set(self.h, layer, kind, ti.type, raw.ctypes.data, ti.n_elements) == 0, name
        self.has_mtp = "mtp.fc.weight" in f.tensors
        self.gemma = arch == "gemma4"
        if self.gemma:
            self.gcfg = gemma_config(md, self.hidden)
            L.or_model_set_gemma(self.h, ctypes.byref(self.gcfg))
        L.or_model_reset(self.h)

    def close(self):
        if self.h:
            self.L.or_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        self.L.or_model_reset(self.h)

    def set_kv_bf16(self, on):
        """round cached keys / values to bf16 as they are written (the engine's
        ifr_ctx_set_kv_bf16 cache); applies to positions written from now on"""
        self.L.or_model_set_kv_bf16(self.h, 1 if on else 0)

    def forward_token(self, token, pos):
        lg = np.empty(self.vocab, np.float32)
        hd = np.empty(self.hidden, np.float32)
        assert self.L.or_forward_token(self.h, int(token), int(pos), _p(lg, _fp), _p(hd, _fp)) == 0
        return lg, hd

    def mtp_step(self, token, hidden, pos):
        lg = np.empty(self.vocab, np.float32)
        ho = np.empty(self.hidden, np.float32)
        hi = np.ascontiguousarray(hidden, np.float32)
        assert self.L.or_mtp_step(self.h, int(token), _p(hi, _fp), int(pos), _p(lg, _fp), _p(ho, _fp)) == 0
        return lg, ho

    def spec_decode(self, prompt, n_steps, gamma, drafts=None):
        """Greedy speculative decoding with the engine's protocol: MTP drafts
        (first from the hidden of the last accepted column, then from the MTP
        layer output), one verify over [last, drafts], longest matching prefix,
        the target's token at the first mismatch, state rolled back to the
        accepted prefix.  drafts: optional callable(step) -> gamma tokens."""
        L = self.L
        self.reset()
        for i, t in enumerate(prompt):
            lg, hid = self.forward_token(t, i)
        last = int(np.argmax(lg))
        out, pos, h = [last], len(prompt), hid
        steps = []
        import time as _time
        for s in range(n_steps):
            t_step = _time.perf_counter()
            if drafts is None:
                ds, hin = [], h
                for j in range(1, gamma + 1):
                    tok = last if j == 1 else ds[-1]
                    dl, hin = self.mtp_step(tok, hin, pos + j - 1)
                    ds.append(int(np.argmax(dl)))
            else:
                ds = [int(x) for x in drafts(s)]
            snap = L.or_snapshot_take(self.h)
            cols = [last] + ds
            lgs, hs = [], []
            for t, tok in enumerate(cols):
                lg, hd = self.forward_token(tok, pos + t)
                lgs.append(lg)
                hs.append(hd)
            acc = 0
            while acc < gamma and int(np.argmax(lgs[acc])) == ds[acc]:
                acc += 1
            y = int(np.argmax(lgs[acc]))
            L.or_snapshot_restore(self.h, snap)
            L.or_snapshot_free(snap)
            for t in range(acc + 1):
                self.forward_token(cols[t], pos + t)
            out += ds[:acc] + [y]
            steps.append(dict(drafts=ds, logits=np.stack(lgs), hidden=np.stack(hs), acc=acc, pos=pos,
                              seconds=_time.perf_counter() - t_step))
            pos += acc + 1
            h = hs[acc]
            last = y
        return out, steps

    def greedy(self, prompt, n_tokens):
        """plain greedy decoding (generate_stream_cpu at temperature 0)"""
        self.reset()
        for i, t in enumerate(prompt):
            lg, _ = self.forward_token(t, i)
        out = [int(np.argmax(lg))]
        pos = len(prompt)
        while len(out) < n_tokens:
            lg, _ = self.forward_token(out[-1], pos)
            pos += 1
            out.append(int(np.argmax(lg)))
        return out
