"""GPU parity of the Gemma4 blocks (config 5's target and draft semantics,
src/Gemma4.jl:253-693) against the CPU oracle's restatement: sliding-window
and full-attention layers (their two RoPE tables), Q/K norms with weights and
the V norm without, attention-logit and final-logit softcaps, GELU-tanh MLP,
the norms after both sub-blocks, the layer scalar and the scaled embedding.
The gemma_mini model has a 6-key window on every other layer, so prompts of
a few dozen tokens already mask most keys of the sliding layers."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4  # exact path, f32 accumulation on both sides


@pytest.fixture(scope="module")
def gmini(pkg, O, ctx):
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model
    path = synth.cached("gemma_mini", seed=1)
    model = Model(ctx, path)
    om = O.OracleModel(gguf.GGUFFile(path), 1100)
    assert om.gemma
    yield path, model, om
    model.free()


def _forced_plan(om, prompt, G, n_steps):
    greedy = om.greedy(list(prompt), 1 + n_steps * (G + 1) + G)

    def drafts(s, emitted):
        d = list(greedy[len(emitted):len(emitted) + G])
        if s % 3 == 1:
            d[1] = (d[1] + 5) % om.vocab
        elif s % 3 == 2:
            d[0] = (d[0] + 5) % om.vocab
        return d
    return greedy, drafts


@pytest.mark.parametrize("P,max_ctx", [(20, 128), (300, 1100)], ids=["cluster", "split_kv"])
def test_gemma_spec_decode_matches_oracle(O, ctx, gmini, P, max_ctx):
    """one request, forced drafts (full accept, a wrong second draft, a wrong
    first draft): tokens equal and verify logits within 1e-4 at every step,
    on the cluster attention kernel (short cache) and the split-KV kernels"""
    from inferno_b200 import synth
    from inferno_b200.engine import State
    _, model, om = gmini
    G, steps = 3, 6
    prompt = synth.prompt(om.vocab, P, seed=P)
    greedy, drafts = _forced_plan(om, prompt, G, steps)
    st = State(model, max_ctx)
    emitted = [int(st.prefill(prompt))]
    assert emitted[0] == greedy[0]
    used, logits = [], []
    for s in range(steps):
        d = drafts(s, emitted)
        used.append(d)
        st.spec_step(G, d)
        logits.append(st.last_verify()[0])
        emitted = [int(t) for t in st.read()[0]]
    assert emitted == greedy[:len(emitted)]
    out, ref = om.spec_decode(list(prompt), steps, G, drafts=lambda s: used[s])
    assert emitted == out
    for s in range(steps):
        err = O.norm_rel(logits[s], ref[s]["logits"]).max()
        assert err < LOGIT_TOL, (s, err)
    # the final softcap bounds every logit
    cap = om.gcfg.final_softcap
    assert cap > 0 and np.abs(np.concatenate(logits)).max() <= cap
    st.free()


def test_gemma_batch_matches_oracle(O, ctx, gmini):
    """three requests in one state (split-KV attention over the batch), exact path"""
    from inferno_b200 import synth
    from inferno_b200.engine import State
    _, model, om = gmini
    B, G, steps = 3, 2, 3
    prompts = np.stack([synth.prompt(om.vocab, 17, seed=40 + b) for b in range(B)])
    plans = [_forced_plan(om, p, G, steps) for p in prompts]
    ctx.set_dense_min_cols(10**6)
    try:
        st = State(model, 128, batch=B)
        firsts = st.prefill(prompts)
        emitted = [[int(firsts[b])] for b in range(B)]
        used = [[] for _ in range(B)]
        logits = []
        for s in range(steps):
            d = np.array([plans[b][1](s, emitted[b]) for b in range(B)], np.int32)
            for b in range(B):
                used[b].append(list(d[b]))
            st.spec_step(G, d)
            logits.append(st.last_verify()[0].reshape(B, G + 1, -1))
            emitted = [[int(t) for t in st.read(b)[0]] for b in range(B)]
        for b in range(B):
            out, ref = om.spec_decode(list(prompts[b]), steps, G, drafts=lambda s: used[b][s])
            assert emitted[b] == out, b
            for s in range(steps):
                assert O.norm_rel(logits[s][b], ref[s]["logits"]).max() < LOGIT_TOL, (b, s)
        st.free()
    finally:
        ctx.set_dense_min_cols(24)


def test_gemma_draft_model_spec_decode(O, ctx, gmini):
    """ifr_spec_step_draft with a Gemma4-block draft model: its greedy tokens
    (argmax of its softcapped logits) are the drafts"""
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model, State
    path, target, om = gmini
    dpath = synth.cached("gemma_mini", seed=2)
    dm = O.OracleModel(gguf.GGUFFile(dpath), 256)
    draft = Model(ctx, dpath)
    prompt = [int(t) for t in synth.prompt(om.vocab, 15, seed=9)]
    G, steps = 3, 4
    ts, ds = State(target, 128), State(draft, 128)
    first = int(ts.prefill(np.array(prompt, np.int32)))
    ds.prefill(np.array(prompt, np.int32))
    plan, out = [], [first]
    for s in range(steps):
        plan.append([int(t) for t in dm.greedy(prompt + out, G)])
        out, _ = om.spec_decode(prompt, s + 1, G, drafts=lambda i: plan[i])
    ref_out, ref = om.spec_decode(prompt, steps, G, drafts=lambda i: plan[i])
    for s in range(steps):
        ts.spec_step_draft(ds, G)
        lg, _, tk = ts.last_verify()
        assert list(tk[1:]) == plan[s], (s, tk, plan[s])
        assert O.norm_rel(lg, ref[s]["logits"]).max() < LOGIT_TOL, s
    assert [int(t) for t in ts.read()[0]] == ref_out
    ts.free()
    ds.free()
    draft.free()


@pytest.fixture(scope="module")
def gpli(pkg, O, ctx):
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model
    path = synth.cached("gemma_pli", seed=1)
    model = Model(ctx, path)
    om = O.OracleModel(gguf.GGUFFile(path), 256)
    assert om.gemma and om.gcfg.pli == 256
    yield path, model, om
    model.free()


def test_gemma_per_layer_inputs_match_oracle(O, ctx, gpli):
    """Gemma4 per-layer inputs (compute_per_layer_inputs! and
    per_layer_input_forward!, Gemma4.jl:459-533): the per-token table rows
    and model projection, and after every MLP block the gated per-layer
    projection before the layer scalar; one request through a 70-token
    prompt (a 64-token prefill chunk and single tokens) and spec steps with
    forced drafts: tokens equal, verify logits within 1e-4"""
    from inferno_b200 import synth
    from inferno_b200.engine import State
    _, model, om = gpli
    G, steps = 3, 5
    prompt = synth.prompt(om.vocab, 70, seed=9)
    greedy, drafts = _forced_plan(om, prompt, G, steps)
    st = State(model, 200)
    emitted = [int(st.prefill(prompt))]
    assert emitted[0] == greedy[0]
    used, logits = [], []
    for s in range(steps):
        d = drafts(s, emitted)
        used.append(d)
        st.spec_step(G, d)
        logits.append(st.last_verify()[0])
        emitted = [int(t) for t in st.read()[0]]
    out, ref = om.spec_decode(list(prompt), steps, G, drafts=lambda s: used[s])
    assert emitted == out
    for s in range(steps):
        err = O.norm_rel(logits[s], ref[s]["logits"]).max()
        assert err < LOGIT_TOL, (s, err)
    st.free()


def test_gemma_per_layer_inputs_batch(O, ctx, gpli):
    """two requests in one state with per-layer inputs, exact path"""
    from inferno_b200 import synth
    from inferno_b200.engine import State
    _, model, om = gpli
    B, G, steps = 2, 2, 3
    prompts = np.stack([synth.prompt(om.vocab, 15, seed=60 + b) for b in range(B)])
    plans = [_forced_plan(om, p, G, steps) for p in prompts]
    ctx.set_dense_min_cols(10**6)
    try:
        st = State(model, 128, batch=B)
        firsts = st.prefill(prompts)
        emitted = [[int(firsts[b])] for b in range(B)]
        used = [[] for _ in range(B)]
        logits = []
        for s in range(steps):
            d = np.array([plans[b][1](s, emitted[b]) for b in range(B)], np.int32)
            for b in range(B):
                used[b].append(list(d[b]))
            st.spec_step(G, d)
            logits.append(st.last_verify()[0].reshape(B, G + 1, -1))
            emitted = [[int(t) for t in st.read(b)[0]] for b in range(B)]
        for b in range(B):
            out, ref = om.spec_decode(list(prompts[b]), steps, G, drafts=lambda s: used[b][s])
            assert emitted[b] == out, b
            for s in range(steps):
                assert O.norm_rel(logits[s][b], ref[s]["logits"]).max() < LOGIT_TOL, (b, s)
        st.free()
    finally:
        ctx.set_dense_min_cols(24)
