"""GPU parity of the fused layer stack (ifr_ctx_set_fused_layers): the decoder
layers of a one-request verify as one persistent cooperative launch, phases
separated by grid barriers.  Same arithmetic as the separate launches
(forward_cpu!, reference src/ModelCPU.jl:976-1020): every verify column's
logits within 1e-4 of the oracle, within 1e-5 of the separate-launch path,
and the same drafts, accept counts and emitted tokens - at config-1 shapes
(Q4_K layers, SSM head dim 128, attention head dim 256), for 1..8 verify
columns, across the split-KV slices of a long cache, and under CUDA-graph
capture."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4   # vs the oracle (f32 accumulation both sides)
PATH_TOL = 5e-5    # fused vs separate launches (same arithmetic, other summation grouping)


@pytest.fixture(scope="module")
def tiny(pkg, ctx):
    from inferno_b200 import synth
    from inferno_b200.engine import Model
    model = Model(ctx, synth.cached("tiny", seed=0))
    yield model
    ctx.set_fused_layers(False)
    model.free()


def _fused_count(st):
    prof, _ = st.profile_read()
    return prof["fused_layers"]["count"]


def _forced(greedy, emitted, G, kind, V):
    d = list(greedy[len(emitted):len(emitted) + G])
    if kind == 1:
        d[min(2, G - 1)] = (d[min(2, G - 1)] + 1) % V
    elif kind == 2:
        d[0] = (d[0] + 1) % V
    return d


def test_fused_config1_matches_oracle_and_separate_launches(O, ctx, tiny):
    """128-token prompt, gamma 4 (5 verify columns), forced drafts: all
    accepted, a wrong third draft, a wrong first draft (SSM replay, conv
    history and KV rollback through the fused launch)"""
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import State
    model = tiny
    V, G = model.info.vocab, 4
    path = synth.cached("tiny", seed=0)
    om = O.OracleModel(gguf.GGUFFile(path), 300)
    prompt = synth.prompt(V, 128, seed=0)
    greedy = om.greedy(list(prompt), 64)
    fa, sep = State(model, 300), State(model, 300)
    e_f = [int(fa.prefill(prompt))]
    e_s = [int(sep.prefill(prompt))]
    plans, lf = [], []
    fa.profile(True)
    for k in [0, 1, 0, 2, 0, 1]:
        d = _forced(greedy, e_f, G, k, V)
        plans.append(d)
        ctx.set_fused_layers(True)
        fa.spec_step(G, d)
        ctx.set_fused_layers(False)
        sep.spec_step(G, d)
        lg_f, hd_f, tk_f = fa.last_verify()
        lg_s, hd_s, tk_s = sep.last_verify()
        assert list(tk_f) == list(tk_s)
        assert O.norm_rel(lg_f, lg_s).max() < PATH_TOL
        assert O.norm_rel(hd_f, hd_s).max() < PATH_TOL
        lf.append(lg_f)
        tf, pf, af, _ = fa.read()
        ts, ps, as_, _ = sep.read()
        assert (pf, af) == (ps, as_) and list(tf) == list(ts)
        e_f = [int(t) for t in tf]
    assert _fused_count(fa) == len(plans)
    out, ref = om.spec_decode(list(prompt), len(plans), G, drafts=lambda s: plans[s])
    assert e_f == out
    for s in range(len(plans)):
        assert O.norm_rel(lf[s], ref[s]["logits"]).max() < LOGIT_TOL, s
    fa.free()
    sep.free()
    om.close()


@pytest.mark.parametrize("G", [0, 1, 3, 7])
def test_fused_every_column_count(ctx, tiny, G):
    """1, 2, 4 and 8 verify columns (one and two column tiles), MTP drafts"""
    from inferno_b200 import synth
    from inferno_b200.engine import State
    model = tiny
    prompt = synth.prompt(model.info.vocab, 40, seed=G + 3)
    fa, sep = State(model, 200), State(model, 200)
    fa.prefill(prompt)
    sep.prefill(prompt)
    fa.profile(True)
    for _ in range(3):
        ctx.set_fused_layers(True)
        fa.spec_step(G)
        ctx.set_fused_layers(False)
        sep.spec_step(G)
        lg_f, _, tk_f = fa.last_verify()
        lg_s, _, tk_s = sep.last_verify()
        assert list(tk_f) == list(tk_s)
        assert lg_f.shape[0] == G + 1
        assert np.abs(lg_f - lg_s).max() / np.abs(lg_s).max() < PATH_TOL
        assert list(fa.read()[0]) == list(sep.read()[0])
    assert _fused_count(fa) == 3
    fa.free()
    sep.free()


def test_fused_long_cache_split_slices(ctx, tiny):
    """a 1400-token prompt: the attention phases spread each KV head's keys
    over many slices and merge them in the combine phase"""
    from inferno_b200 import synth
    from inferno_b200.engine import State
    model = tiny
    prompt = synth.prompt(model.info.vocab, 1400, seed=11)
    fa, sep = State(model, 1500), State(model, 1500)
    fa.prefill(prompt)
    sep.prefill(prompt)
    fa.profile(True)
    for _ in range(4):
        ctx.set_fused_layers(True)
        fa.spec_step(4)
        ctx.set_fused_layers(False)
        sep.spec_step(4)
        lg_f, _, tk_f = fa.last_verify()
        lg_s, _, tk_s = sep.last_verify()
        assert list(tk_f) == list(tk_s)
        assert np.abs(lg_f - lg_s).max() / np.abs(lg_s).max() < PATH_TOL
    assert list(fa.read()[0]) == list(sep.read()[0])
    assert _fused_count(fa) == 4
    fa.free()
    sep.free()


def test_fused_graph_capture(pkg, ctx, tiny):
    """spec steps captured as a CUDA graph with the fused launch (counter reset
    and cooperative launch inside the graph) replay to the eager tokens"""
    import torch
    from inferno_b200 import synth
    from inferno_b200.engine import Model, State
    c2 = pkg.Context(0, torch_stream=False)
    try:
        model = Model(c2, synth.cached("tiny", seed=0))
        prompt = synth.prompt(model.info.vocab, 64, seed=21)
        g, e = State(model, 300), State(model, 300)
        g.prefill(prompt)
        e.prefill(prompt)
        c2.set_fused_layers(True)
        g.spec_step(4)
        g.capture(4, 3)
        for _ in range(2):
            g.launch()
        c2.set_fused_layers(False)
        for _ in range(7):
            e.spec_step(4)
        c2.sync()
        assert list(g.read()[0]) == list(e.read()[0])
        lg_g, _, _ = g.last_verify()
        lg_e, _, _ = e.last_verify()
        assert np.abs(lg_g - lg_e).max() / np.abs(lg_e).max() < PATH_TOL
        g.free()
        e.free()
        model.free()
    finally:
        torch.cuda.synchronize()
        c2.close()


def test_fused_barrier_timeout_reported_and_context_usable(O, pkg, ctx, tiny):
    """failure detection without a fault: one CTA of a fused launch leaves
    without arriving at the grid barrier; the others' bounded waits (~2 s)
    run out, the launch returns, ifr_sync reports IFR_ERR_TIMEOUT, and the
    context then runs a fused spec step that matches the separate launches"""
    from inferno_b200 import _lib, synth
    from inferno_b200.engine import State
    rc = _lib.load().ifr_test_fused_timeout(ctx.handle)
    assert rc == _lib.IFR_ERR_TIMEOUT, rc
    ctx.sync()  # the error flag was read and cleared
    prompt = synth.prompt(tiny.info.vocab, 24, seed=77)
    fa, sep = State(tiny, 128), State(tiny, 128)
    fa.prefill(prompt)
    sep.prefill(prompt)
    ctx.set_fused_layers(True)
    fa.spec_step(4)
    ctx.set_fused_layers(False)
    sep.spec_step(4)
    lg_f, _, tk_f = fa.last_verify()
    lg_s, _, tk_s = sep.last_verify()
    assert list(tk_f) == list(tk_s)
    assert np.abs(lg_f - lg_s).max() / np.abs(lg_s).max() < PATH_TOL
    fa.free()
    sep.free()
