"""CPU tests of the oracle against the golden fixtures and the reference's
known answers (no GPU).  The oracle is the checker for every GPU parity test,
so it is pinned here first."""
import json
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FORMATS = [("Q4_K", 12), ("Q5_K", 13), ("Q6_K", 14), ("Q8_0", 8)]


@pytest.mark.parametrize("name,qt", FORMATS)
def test_dequant_bit_exact_vs_gguf_py(O, name, qt):
    """64 random valid blocks: bit-exact with gguf-py 0.19.0's dequantize."""
    g = np.load(os.path.join(GOLD, "dequant_golden.npz"))
    be, _ = O.BLOCK[qt]
    got = O.dequantize(qt, g[f"{name}_blocks"], 64 * be)
    assert np.array_equal(got.view(np.uint32), g[f"{name}_gguf_py"].view(np.uint32))


@pytest.mark.parametrize("name,qt", FORMATS)
def test_dequant_known_answer(O, name, qt):
    """hand-built blocks with d = 1.0 (f16 0x3c00): values written out by hand"""
    g = np.load(os.path.join(GOLD, "dequant_golden.npz"))
    be, _ = O.BLOCK[qt]
    got = O.dequantize(qt, g[f"{name}_ka_block"], be)
    assert np.array_equal(got, g[f"{name}_ka_expected"])


@pytest.mark.parametrize("name,qt", FORMATS)
def test_gemv_vs_reference_c_kernel(O, name, qt):
    """Oracle GEMV (Q8_K activations for the K-quants, f32 for Q8_0, as the
    reference's kernels) against outputs of the reference's own
    quant_kernels.c: equal up to the C kernel's f32 accumulation order."""
    g = np.load(os.path.join(GOLD, "gemv_golden.npz"))
    M, K = int(g["M"]), int(g["K"])
    Y = O.gemm_ref(qt, g[f"{name}_W"], M, K, g["X"], act=1)
    assert O.norm_rel(g[f"{name}_ref"], Y).max() < 1e-5
    if qt != 8:  # f32 activations differ from the reference's quantized ones
        assert O.norm_rel(g[f"{name}_ref"], O.gemm_f64(qt, g[f"{name}_W"], M, K, g["X"])).max() > 1e-4


def test_q8k_activations_differ_from_exact(O):
    """Q8_K activation rounding moves a GEMV by ~1e-2 (why the engine keeps
    exact activations by default)"""
    rng = np.random.default_rng(4)
    for qt in (12, 13, 14):
        M, K = 64, 2048
        q = O.quantize(qt, rng.normal(0, 0.02, (M, K)).astype(np.float32))
        X = rng.normal(0, 1, (3, K)).astype(np.float32)
        err = O.norm_rel(O.gemm_q8k(qt, q, M, K, X), O.gemm_f64(qt, q, M, K, X)).max()
        assert 1e-3 < err < 3e-2


def test_quantize_q8k_vs_reference(O):
    """the Q8_K restatement against quantize_row_q8_K of the reference (built
    from its sources into oracle/_ref when the reference tree is present)"""
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 4096).astype(np.float32)
    x[256:512] *= 1e-3
    x[512:768] = 0.0
    x[768 + 17] = 50.0
    d, q = O.quantize_q8k(x)
    assert d[2] == 0.0 and not q[512:768].any()
    assert np.abs(q).max() == 127
    np.testing.assert_allclose(np.repeat(d, 256) * q, x, atol=float(d.max()) * 0.5 + 1e-12)
    R = O.ref_quantize_q8k(x) if hasattr(O, "ref_quantize_q8k") else None
    if R is None:
        pytest.skip("oracle/_ref not built")
    assert np.array_equal(R[0], d) and np.array_equal(R[1], q)


def test_gemv_f32_vs_f64(O):
    rng = np.random.default_rng(1)
    M, K = 64, 2048
    q = O.quantize(12, rng.normal(0, 0.02, (M, K)).astype(np.float32))
    X = rng.normal(0, 1, (3, K)).astype(np.float32)
    assert O.norm_rel(O.gemm_f32(12, q, M, K, X), O.gemm_f64(12, q, M, K, X)).max() < 1e-5


@pytest.mark.parametrize("name,qt", FORMATS)
def test_encoder_round_trip(O, name, qt):
    """own encoder: dequant(quant(w)) close to w, and re-encoding is stable"""
    rng = np.random.default_rng(2)
    w = rng.normal(0, 0.02, (8, 512)).astype(np.float32)
    q = O.quantize(qt, w)
    assert q.size == 8 * O.row_bytes(qt, 512)
    d = O.dequantize(qt, q, w.size).reshape(w.shape)
    rel = np.linalg.norm(d - w) / np.linalg.norm(w)
    assert rel < {12: 0.1, 13: 0.05, 14: 0.03, 8: 0.01}[qt]


def test_f16_conversion(O):
    L = O.lib()
    vals = np.array([0.0, 1.0, -2.5, 65504.0, 6.1035156e-05, 5.96e-08, 1e-9, 70000.0, 0.1],
                    np.float32)
    for v in vals:
        assert L.or_f32_to_f16(float(v)) == int(np.float16(v).view(np.uint16))
    for h in range(0, 0x7c00, 37):
        assert L.or_f16_to_f32(h) == float(np.uint16(h).view(np.float16))


def test_sample_from_probs_known_answers(O):
    """tests/unit/test_speculative_decoding.jl:13-46 of the reference: the
    answers hold for every draw r in (0, 1)"""
    g = json.load(open(os.path.join(GOLD, "sampler_golden.json")))
    for case in g["sample_from_probs"]:
        for r in (1e-6, 0.3, 0.999):
            assert O.sample_from_probs(case["probs"], r) == case["expect"]


def test_exp_accuracy(O):
    xs = np.concatenate([np.linspace(-87, 0, 4001), np.linspace(0, 88, 2001)]).astype(np.float32)
    got = np.array([O.exp(v) for v in xs], np.float64)
    ref = np.exp(xs.astype(np.float64))
    assert np.max(np.abs(got - ref) / ref) < 2e-7
    assert O.exp(-100.0) == 0.0


def _softmax(x, T):
    z = (x - x.max()) / T
    e = np.exp(z.astype(np.float64))
    return e / e.sum()


def test_accept_distribution_matches_target(O):
    """Rejection sampling property: with drafts drawn from p_d, the first
    emitted token is distributed as p_t (exact algorithm, tiny vocab)."""
    rng = np.random.default_rng(3)
    V, T, n = 6, 0.8, 40000
    tl = rng.normal(0, 1.5, V).astype(np.float32)
    dl = (tl + rng.normal(0, 1.0, V)).astype(np.float32)
    tgt = np.broadcast_to(np.stack([tl, tl]), (n, 2, V)).copy()
    dft = np.broadcast_to(dl, (n, 1, V)).copy()
    u = rng.random((n, 3), dtype=np.float32)
    acc, out, dtok = O.accept(tgt, dft, u, T)
    first = out[:, 0]
    emp = np.bincount(first, minlength=V) / n
    pt = _softmax(tl, T)
    assert np.abs(emp - pt).max() < 0.01
    # drafts follow p_d
    pd = _softmax(dl, T)
    assert np.abs(np.bincount(dtok[:, 0], minlength=V) / n - pd).max() < 0.01
    # accept rate = sum min(p_t, p_d)
    assert abs(acc.mean() - np.minimum(pt, pd).sum()) < 0.01


def test_accept_identical_distributions_accepts_all(O):
    rng = np.random.default_rng(4)
    B, G, V = 8, 4, 3000
    tgt = rng.normal(0, 3, (B, G + 1, V)).astype(np.float32)
    dft = tgt[:, :G].copy()
    u = rng.random((B, 2 * G + 1), dtype=np.float32) * 0.999
    acc, out, d = O.accept(tgt, dft, u, 0.8)
    assert (acc == G).all()
    assert (out[:, :G] == d).all() and (out[:, G] >= 0).all()


def test_accept_greedy_semantics(O):
    B, G, V = 3, 3, 10
    tgt = np.zeros((B, G + 1, V), np.float32)
    am = np.array([[1, 2, 3, 4], [1, 5, 3, 4], [7, 7, 7, 7]])
    for b in range(B):
        for i in range(G + 1):
            tgt[b, i, am[b, i]] = 1.0
    drafts = np.array([[1, 2, 3], [1, 2, 3], [0, 7, 7]], np.int32)
    acc, out = O.accept_greedy(tgt, drafts)
    assert acc.tolist() == [3, 1, 0]
    assert out[0].tolist() == [1, 2, 3, 4]
    assert out[1].tolist() == [1, 5, -1, -1]
    assert out[2].tolist() == [7, -1, -1, -1]


def test_argmax_ties_first_index(O):
    L = O.lib()
    import ctypes
    a = np.array([0.0, 2.0, 1.0, 2.0], np.float32)
    assert L.or_argmax(a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), 4) == 1


@pytest.mark.parametrize("qt", [12, 13, 14, 8])
def test_oracle_encoder_matches_library(O, pkg, qt):
    """the oracle's GGUF encoder writes the library's bytes, so the CPU
    reference arm of bench.py can build the seeded model without loading
    libinferno_b200.so and still run the same model as the GPU arm"""
    rng = np.random.default_rng(11 + qt)
    for std in (0.02, 0.5, 3.0):
        x = (rng.standard_normal((48, 1024)) * std).astype(np.float32)
        assert np.array_equal(O.quantize(qt, x), pkg.quantize(qt, x))


def test_synth_model_same_bytes_with_oracle_encoder(O, pkg, tmp_path):
    from inferno_b200 import synth
    a = synth.build(str(tmp_path / "lib.gguf"), "mini", 3)
    b = synth.build(str(tmp_path / "oracle.gguf"), "mini", 3, quantize=O.quantize)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_gemma_oracle_blocks(O, pkg, tmp_path):
    """the oracle's Gemma4 restatement on the small Gemma4-block model: the
    final softcap bounds every logit, the embedding scale is sqrt(hidden),
    and the forward is deterministic across a reset"""
    from inferno_b200 import synth, gguf
    path = synth.build(str(tmp_path / "g.gguf"), "gemma_mini", 1, quantize=O.quantize)
    om = O.OracleModel(gguf.GGUFFile(path), 64)
    assert om.gemma and om.gcfg.window == 6 and om.gcfg.sliding_pattern == 2
    assert om.gcfg.embed_scale == np.float32(16.0)
    prompt = synth.prompt(om.vocab, 20, seed=2)
    a = om.greedy(list(prompt), 6)
    b = om.greedy(list(prompt), 6)
    assert a == b
    lg, _ = om.forward_token(a[-1], len(prompt) + 5)
    assert np.isfinite(lg).all() and np.abs(lg).max() <= om.gcfg.final_softcap


def test_gemma_oracle_per_layer_inputs_first_token(O, pkg, tmp_path):
    """the oracle's Gemma4 per-layer inputs against an independent numpy
    restatement of forward! for the first token (Gemma4.jl:459-533, 604-676):
    at position 0 every attention head sees one key, so the block reduces to
    norms and projections and the whole layer stack is a few matrix products"""
    from inferno_b200 import synth, gguf
    path = synth.build(str(tmp_path / "p.gguf"), "gemma_pli", 1, quantize=O.quantize)
    f = gguf.GGUFFile(path)
    om = O.OracleModel(f, 16)
    cfg = om.gcfg
    assert cfg.pli == 256
    d, L, P = om.hidden, om.cfg.n_layers, cfg.pli
    nh, nkv, hd = om.cfg.n_head, om.cfg.n_kv_head, om.cfg.head_dim
    eps = np.float32(om.cfg.rms_eps)

    def W(name):
        ti = f.tensors[name]
        v = O.dequantize(ti.type, np.ascontiguousarray(f.raw(name)), ti.n_elements).astype(np.float64)
        return v.reshape(list(reversed(ti.dims))) if len(ti.dims) == 2 else v

    def rms(x, w):
        return x / np.sqrt(np.mean(x * x) + eps) * w

    def gelu(x):
        c = np.sqrt(2.0 / np.pi)
        return 0.5 * x * (1.0 + np.tanh(c * (x + 0.044715 * x ** 3)))

    tok = 123
    x = W("token_embd.weight")[tok] * np.float64(cfg.embed_scale)
    proj = W("pli_model_proj.weight") @ x
    row = W("pli_token_embd.weight")[tok]
    pli = np.empty(L * P)
    for i in range(L):
        s = slice(i * P, (i + 1) * P)
        pli[s] = (rms(proj[s], W("pli_proj_norm.weight")) + row[s] * np.sqrt(P)) * 2.0 ** -0.5
    for i in range(L):
        pre = f"blk.{i}."
        xn = rms(x, W(pre + "attn_norm.weight"))
        v = (W(pre + "attn_v.weight") @ xn).reshape(nkv, hd)
        v = v / np.sqrt(np.mean(v * v, axis=1, keepdims=True) + eps)  # V norm without weights
        o = np.repeat(v, nh // nkv, axis=0).reshape(-1)  # one key: softmax weight 1
        x = x + rms(W(pre + "attn_output.weight") @ o, W(pre + "post_attention_norm.weight"))
        xn = rms(x, W(pre + "ffn_norm.weight"))
        h = gelu(W(pre + "ffn_gate.weight") @ xn) * (W(pre + "ffn_up.weight") @ xn)
        x = x + rms(W(pre + "ffn_down.weight") @ h, W(pre + "post_ffw_norm.weight"))
        g = gelu(W(pre + "pli_gate.weight") @ x) * pli[i * P:(i + 1) * P]
        x = x + rms(W(pre + "pli_proj.weight") @ g, W(pre + "pli_post_norm.weight"))
        x = x * W(pre + "layer_scalar")[0]
    hid = rms(x, W("output_norm.weight"))
    _, hd_o = om.forward_token(tok, 0)
    assert O.norm_rel(hd_o.reshape(1, -1), hid.reshape(1, -1)).max() < 1e-5
