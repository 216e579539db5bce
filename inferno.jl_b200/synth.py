"""Seeded synthetic Qwen3.5-hybrid GGUF models (no checkpoints are available).

Presets follow the benchmark configurations:
  tiny  hidden 1024, 24 layers (attention every 4th), 8 q / 2 kv heads x 256,
        partial RoPE 25%, SSM 16 heads x 128 (inner 2048, conv kernel 4),
        FFN 3584, vocab 151936; Q4_K matmuls, Q6_K tied embedding / lm_head,
        F32 norms; one-layer MTP draft head
  9b    hidden 4096, 32 layers, 16 q / 4 kv heads x 256, SSM 32 heads x 128,
        FFN 12288, vocab 151936; Q4_K matmuls, Q6_K ffn_down and lm_head
  mini  a small model of the same structure for fast tests
  9b_narrow, gemma_narrow  the large configs' widths with 4 / 2 layers (parity)
Weights are N(0, 0.02) (the layer norms, which GGUF stores as 1 + w, are
1 + N(0, 0.02); ssm_a = -exp(N(0, 0.5)); conv1d N(0, 0.5)), quantized with the
library's own encoder.  Presets with `row_pool` (9b) draw that many rows per
matrix and repeat them down the matrix, so that the 5 GB model is built in
seconds; the bytes per weight and the kernels' work are unchanged.  Tensor names and metadata keys are those the
reference's loader reads (src/LoaderCPU.jl:439-694).
"""
import os
import tempfile

import numpy as np

from . import gguf as G

PRESETS = {
    "tiny": dict(hidden=1024, n_layers=24, n_head=8, n_kv_head=2, head_dim=256, rope_frac=0.25,
                 ffn=3584, vocab=151936, ssm_heads=16, ssm_head_dim=128, conv_kernel=4,
                 attn_every=4, mat=G.GGML_Q4_K, down=G.GGML_Q4_K, emb=G.GGML_Q6_K, mtp=True,
                 context=4096),
    "9b": dict(hidden=4096, n_layers=32, n_head=16, n_kv_head=4, head_dim=256, rope_frac=0.25,
               ffn=12288, vocab=151936, ssm_heads=32, ssm_head_dim=128, conv_kernel=4,
               attn_every=4, mat=G.GGML_Q4_K, down=G.GGML_Q6_K, emb=G.GGML_Q6_K, mtp=True,
               context=8192, row_pool=1024),
    "mini": dict(hidden=256, n_layers=4, n_head=4, n_kv_head=2, head_dim=64, rope_frac=0.25,
                 ffn=512, vocab=4096, ssm_heads=4, ssm_head_dim=64, conv_kernel=4,
                 attn_every=4, mat=G.GGML_Q4_K, down=G.GGML_Q4_K, emb=G.GGML_Q6_K, mtp=True,
                 context=4096),
    # config 5: the Gemma4-shape target (hidden 5376, 62 layers, 32 q / 16 kv x
    # 128, FFN 21504, vocab 262144, Q4_K) and its Q8_0 draft model (hidden
    # 1152, 26 layers), both with Gemma4 blocks (architecture "gemma4"): five
    # sliding-window layers to one full layer, GELU-tanh MLP, Q/K/V norms,
    # norms around both blocks, a layer scalar, attention and final logit
    # softcaps, the embedding scaled by sqrt(hidden)
    "gemma": dict(arch="gemma4", hidden=5376, n_layers=62, n_head=32, n_kv_head=16, head_dim=128, rope_frac=0.25,
                  ffn=21504, vocab=262144, ssm_heads=0, ssm_head_dim=0, conv_kernel=4,
                  attn_every=1, mat=G.GGML_Q4_K, down=G.GGML_Q4_K, emb=G.GGML_Q4_K, mtp=False,
                  context=8192, row_pool=1024, window=1024, pattern=6),
    "gemma_draft": dict(arch="gemma4", hidden=1152, n_layers=26, n_head=4, n_kv_head=1, head_dim=256,
                        rope_frac=0.25, ffn=6912, vocab=262144, ssm_heads=0, ssm_head_dim=0, conv_kernel=4,
                        attn_every=1, mat=G.GGML_Q8_0, down=G.GGML_Q8_0, emb=G.GGML_Q8_0, mtp=False,
                        context=8192, row_pool=1024, window=1024, pattern=6),
    # parity models at the large configs' widths with few layers, so the CPU
    # oracle can follow them: 9b_narrow keeps every width of "9b" (the batched
    # SSM kernel at head dim 128, attention at head dim 256, FFN 12288, Q6_K
    # down) with 3 SSM layers + 1 attention layer; gemma_narrow keeps the
    # Gemma4-shape target's widths with 2 layers and a 32768-token vocabulary
    "9b_narrow": dict(hidden=4096, n_layers=4, n_head=16, n_kv_head=4, head_dim=256, rope_frac=0.25,
                      ffn=12288, vocab=151936, ssm_heads=32, ssm_head_dim=128, conv_kernel=4,
                      attn_every=4, mat=G.GGML_Q4_K, down=G.GGML_Q6_K, emb=G.GGML_Q6_K, mtp=True,
                      context=8192, row_pool=1024),
    "gemma_narrow": dict(arch="gemma4", hidden=5376, n_layers=2, n_head=32, n_kv_head=16, head_dim=128,
                         rope_frac=0.25, ffn=21504, vocab=32768, ssm_heads=0, ssm_head_dim=0, conv_kernel=4,
                         attn_every=1, mat=G.GGML_Q4_K, down=G.GGML_Q4_K, emb=G.GGML_Q4_K, mtp=False,
                         context=8192, row_pool=1024, window=8, pattern=2, attn_cap=20.0, final_cap=2.0),
    # a small Gemma4-block model: the sliding window (6 keys) and both layer
    # kinds within a short prompt, split-KV attention reachable at 1024 tokens
    "gemma_mini": dict(arch="gemma4", hidden=256, n_layers=4, n_head=4, n_kv_head=2, head_dim=128,
                       rope_frac=0.25, ffn=512, vocab=4096, ssm_heads=0, ssm_head_dim=0, conv_kernel=4,
                       attn_every=1, mat=G.GGML_Q4_K, down=G.GGML_Q4_K, emb=G.GGML_Q6_K, mtp=False,
                       context=2048, window=6, pattern=2, attn_cap=10.0, final_cap=1.0),
    # gemma_mini with Gemma4 per-layer inputs (256 per layer)
    "gemma_pli": dict(arch="gemma4", hidden=256, n_layers=4, n_head=4, n_kv_head=2, head_dim=128,
                      rope_frac=0.25, ffn=512, vocab=4096, ssm_heads=0, ssm_head_dim=0, conv_kernel=4,
                      attn_every=1, mat=G.GGML_Q4_K, down=G.GGML_Q4_K, emb=G.GGML_Q6_K, mtp=False,
                      context=2048, window=6, pattern=2, attn_cap=10.0, final_cap=1.0, pli=256,
                      pli_emb=G.GGML_Q8_0),
    # attention-only test model whose heads and FFN units split over 2 ranks
    "tp_mini": dict(hidden=256, n_layers=4, n_head=8, n_kv_head=4, head_dim=64, rope_frac=0.25,
                    ffn=1024, vocab=4096, ssm_heads=0, ssm_head_dim=0, conv_kernel=4,
                    attn_every=1, mat=G.GGML_Q4_K, down=G.GGML_Q4_K, emb=G.GGML_Q6_K, mtp=False,
                    context=1024),
}


def _quant(qtype, x):
    from . import quantize
    return quantize(qtype, x)


def build(path, preset="tiny", seed=0, quantize=None, **overrides):
    """Write the seeded model to `path` (GGUF v3).  `quantize(qtype, rows)`
    encodes the matrices (default: the library's host encoder; the CPU
    reference leg passes the oracle's, which writes the same bytes, so that
    it never loads the library)."""
    quant = quantize or _quant
    cfg = dict(PRESETS[preset])
    cfg.update(overrides)
    d, L = cfg["hidden"], cfg["n_layers"]
    nh, nkv, hd = cfg["n_head"], cfg["n_kv_head"], cfg["head_dim"]
    H, sd = cfg["ssm_heads"], cfg["ssm_head_dim"]
    inner = H * sd
    C = inner + 2 * H * sd
    K = cfg["conv_kernel"]
    ffn, V = cfg["ffn"], cfg["vocab"]
    root = np.random.default_rng(seed)
    w = G.GGUFWriter(path)
    if cfg.get("arch") == "gemma4":
        return _build_gemma(w, cfg, preset, seed, root, quant)
    arch = "qwen35"
    w.add("general.architecture", arch)
    w.add("general.name", f"inferno-b200 synthetic {preset} seed {seed}")
    for k, v in [("embedding_length", d), ("feed_forward_length", ffn), ("block_count", L),
                 ("attention.head_count", nh), ("attention.head_count_kv", nkv),
                 ("attention.key_length", hd), ("attention.value_length", hd),
                 ("context_length", cfg["context"]), ("full_attention_interval", cfg["attn_every"]),
                 ("ssm.inner_size", inner), ("ssm.state_size", sd), ("ssm.group_count", H),
                 ("ssm.time_step_rank", H), ("ssm.conv_kernel", K)]:
        w.add(f"{arch}.{k}", int(v))
    w.add(f"{arch}.attention.layer_norm_rms_epsilon", 1e-6)
    w.add(f"{arch}.rope.freq_base", 10000000.0)
    w.add(f"{arch}.rope.partial_rotary_factor", float(cfg["rope_frac"]))

    def rng():
        return np.random.default_rng(root.integers(1 << 62))

    pool = cfg.get("row_pool", 0)

    def mat(name, rows, cols, qtype, std=0.02):
        n = min(rows, pool) if pool else rows
        x = rng().standard_normal((n, cols), dtype=np.float32) * np.float32(std)
        q = quant(qtype, x)
        if n < rows:  # quantization is row-wise: repeat the quantized rows
            q = np.tile(q.reshape(n, -1), ((rows + n - 1) // n, 1))[:rows].ravel()
        w.add_tensor(name, [cols, rows], qtype, q)

    def f32(name, dims, values):
        w.add_tensor(name, dims, G.GGML_F32, np.ascontiguousarray(values, dtype=np.float32))

    def norm(name, n):
        f32(name, [n], 1.0 + 0.02 * rng().standard_normal(n, dtype=np.float32))

    def attn_layer(pre):
        mat(pre + "attn_q.weight", 2 * nh * hd, d, cfg["mat"])
        mat(pre + "attn_k.weight", nkv * hd, d, cfg["mat"])
        mat(pre + "attn_v.weight", nkv * hd, d, cfg["mat"])
        mat(pre + "attn_output.weight", d, nh * hd, cfg["mat"])
        norm(pre + "attn_q_norm.weight", hd)
        norm(pre + "attn_k_norm.weight", hd)

    def mlp(pre):
        mat(pre + "ffn_gate.weight", ffn, d, cfg["mat"])
        mat(pre + "ffn_up.weight", ffn, d, cfg["mat"])
        mat(pre + "ffn_down.weight", d, ffn, cfg["down"])

    mat("token_embd.weight", V, d, cfg["emb"])
    norm("output_norm.weight", d)
    for i in range(L):
        pre = f"blk.{i}."
        norm(pre + "attn_norm.weight", d)
        norm(pre + "post_attention_norm.weight", d)
        if (i + 1) % cfg["attn_every"] == 0:
            attn_layer(pre)
        else:
            mat(pre + "attn_qkv.weight", C, d, cfg["mat"])
            mat(pre + "attn_gate.weight", inner, d, cfg["mat"])
            mat(pre + "ssm_out.weight", d, inner, cfg["mat"])
            f32(pre + "ssm_conv1d.weight", [K, C], 0.5 * rng().standard_normal((C, K), dtype=np.float32))
            f32(pre + "ssm_alpha.weight", [d, H], 0.02 * rng().standard_normal((H, d), dtype=np.float32))
            f32(pre + "ssm_beta.weight", [d, H], 0.02 * rng().standard_normal((H, d), dtype=np.float32))
            f32(pre + "ssm_a", [H], -np.exp(0.5 * rng().standard_normal(H)).astype(np.float32))
            f32(pre + "ssm_dt.bias", [H], 0.02 * rng().standard_normal(H, dtype=np.float32))
            norm(pre + "ssm_norm.weight", sd)
        mlp(pre)
    if cfg["mtp"]:
        mat("mtp.fc.weight", d, 2 * d, cfg["mat"])
        norm("mtp.pre_fc_norm_embedding.weight", d)
        norm("mtp.pre_fc_norm_hidden.weight", d)
        norm("mtp.norm.weight", d)
        pre = "mtp.blk.0."
        norm(pre + "attn_norm.weight", d)
        norm(pre + "post_attention_norm.weight", d)
        attn_layer(pre)
        mlp(pre)
    w.write()
    return path


def _build_gemma(w, cfg, preset, seed, root, quant):
    """a Gemma4-block model (src/Gemma4.jl): attention-only layers, every
    `pattern`-th a full-attention layer and the others sliding-window ones;
    q rows n_head x head_dim (no output gate); norms stored as their weights
    (no 1 + w offset, CommonOps.rmsnorm! multiplies by w)"""
    d, L = cfg["hidden"], cfg["n_layers"]
    nh, nkv, hd = cfg["n_head"], cfg["n_kv_head"], cfg["head_dim"]
    ffn, V = cfg["ffn"], cfg["vocab"]
    arch = "gemma4"
    w.add("general.architecture", arch)
    w.add("general.name", f"inferno-b200 synthetic {preset} seed {seed}")
    for k, v in [("embedding_length", d), ("feed_forward_length", ffn), ("block_count", L),
                 ("attention.head_count", nh), ("attention.head_count_kv", nkv),
                 ("attention.key_length", hd), ("attention.value_length", hd),
                 ("context_length", cfg["context"]), ("attention.sliding_window", cfg["window"]),
                 ("attention.sliding_window_pattern", cfg["pattern"])]:
        w.add(f"{arch}.{k}", int(v))
    w.add(f"{arch}.attention.layer_norm_rms_epsilon", 1e-6)
    w.add(f"{arch}.rope.freq_base", 1000000.0)
    w.add(f"{arch}.rope.freq_base_swa", 10000.0)
    w.add(f"{arch}.rope.partial_rotary_factor", float(cfg["rope_frac"]))
    w.add(f"{arch}.attn_logit_softcapping", float(cfg.get("attn_cap", 50.0)))
    w.add(f"{arch}.final_logit_softcapping", float(cfg.get("final_cap", 30.0)))
    P = int(cfg.get("pli", 0))
    if P:
        w.add(f"{arch}.embedding_length_per_layer_input", P)

    def rng():
        return np.random.default_rng(root.integers(1 << 62))

    pool = cfg.get("row_pool", 0)

    def mat(name, rows, cols, qtype, std=0.02):
        n = min(rows, pool) if pool else rows
        x = rng().standard_normal((n, cols), dtype=np.float32) * np.float32(std)
        q = quant(qtype, x)
        if n < rows:
            q = np.tile(q.reshape(n, -1), ((rows + n - 1) // n, 1))[:rows].ravel()
        w.add_tensor(name, [cols, rows], qtype, q)

    def f32(name, dims, values):
        w.add_tensor(name, dims, G.GGML_F32, np.ascontiguousarray(values, dtype=np.float32))

    def norm(name, n):
        f32(name, [n], 1.0 + 0.02 * rng().standard_normal(n, dtype=np.float32))

    mat("token_embd.weight", V, d, cfg["emb"])
    norm("output_norm.weight", d)
    for i in range(L):
        pre = f"blk.{i}."
        for nm in ("attn_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm"):
            norm(pre + nm + ".weight", d)
        mat(pre + "attn_q.weight", nh * hd, d, cfg["mat"])
        mat(pre + "attn_k.weight", nkv * hd, d, cfg["mat"])
        mat(pre + "attn_v.weight", nkv * hd, d, cfg["mat"])
        mat(pre + "attn_output.weight", d, nh * hd, cfg["mat"])
        norm(pre + "attn_q_norm.weight", hd)
        norm(pre + "attn_k_norm.weight", hd)
        mat(pre + "ffn_gate.weight", ffn, d, cfg["mat"])
        mat(pre + "ffn_up.weight", ffn, d, cfg["mat"])
        mat(pre + "ffn_down.weight", d, ffn, cfg["down"])
        f32(pre + "layer_scalar", [1], [1.0 + 0.05 * float(rng().standard_normal())])
        if P:
            # per-layer input block: gate (P x d), projection (d x P), post norm
            mat(pre + "pli_gate.weight", P, d, cfg["mat"])
            mat(pre + "pli_proj.weight", d, P, cfg["mat"])
            norm(pre + "pli_post_norm.weight", d)
    if P:
        # the token table (vocab x L P), the model projection (L P x d, stored
        # already scaled by d^-1/2, as the reference scales it at load) and its norm
        mat("pli_token_embd.weight", V, L * P, cfg.get("pli_emb", cfg["emb"]))
        mat("pli_model_proj.weight", L * P, d, cfg["mat"], std=0.02 / float(np.sqrt(d)))
        norm("pli_proj_norm.weight", P)
    w.write()
    return w.path


def cached(preset="tiny", seed=0, directory=None, quantize=None):
    """Path of the seeded model, built on first use (per machine); `quantize`
    as in build()."""
    directory = directory or os.path.join(tempfile.gettempdir(), "inferno_b200_models")
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"{preset}_seed{seed}.gguf")
    if not os.path.exists(path):
        tmp = path + f".{os.getpid()}.tmp"
        build(tmp, preset, seed, quantize=quantize)
        os.replace(tmp, path)
    return path


def prompt(vocab, n=128, seed=0):
    """seeded uniform prompt token ids"""
    return np.random.default_rng(seed + 1_000_003).integers(0, vocab, n).astype(np.int32)
