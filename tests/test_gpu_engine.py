"""GPU parity of the speculative-decoding verify engine against the CPU oracle
(forward_cpu! + MTP head restated in C): draft tokens, verify-column logits,
accept counts and emitted tokens, through the C ABI."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4  # norm-relative per verify column (f32 accumulation both sides)


@pytest.fixture(scope="module")
def mini(pkg, O, ctx):
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model
    path = synth.cached("mini", seed=1)
    model = Model(ctx, path)
    om = O.OracleModel(gguf.GGUFFile(path), 512)
    return model, om, synth.prompt(model.info.vocab, 24, seed=1)


def _state(model, n=512):
    from inferno_b200.engine import State
    return State(model, n)


def test_model_info(mini):
    model, om, _ = mini
    i = model.info
    assert (i.hidden, i.n_layers, i.n_head, i.n_kv_head, i.head_dim, i.rotary_dim) == (256, 4, 4, 2, 64, 16)
    assert (i.ssm_heads, i.ssm_head_dim, i.vocab, i.n_attention_layers, i.has_mtp) == (4, 64, 4096, 1, 1)


def test_spec_decode_mtp_matches_oracle(O, mini):
    model, om, prompt = mini
    G, steps = 4, 6
    st = _state(model)
    first = st.prefill(prompt)
    out_o, ref = om.spec_decode(prompt, steps, G)
    assert first == out_o[0]
    for s in range(steps):
        st.spec_step(G)
        lg, hd, tk = st.last_verify()
        r = ref[s]
        assert list(tk[1:]) == r["drafts"], (s, tk, r["drafts"])
        err = O.norm_rel(lg, r["logits"])
        assert err.max() < LOGIT_TOL, (s, err)
        assert O.norm_rel(hd, r["hidden"]).max() < LOGIT_TOL
        toks, pos, acc, nst = st.read()
        assert acc == r["acc"] and nst == s + 1 and pos == r["pos"] + acc + 1
    toks, *_ = st.read()
    assert list(toks) == out_o


def test_forced_drafts_full_partial_and_rejected(O, mini):
    """drafts from the greedy continuation: all accepted, then one wrong in the
    middle, then a wrong first draft (rollback of SSM, conv and KV state)"""
    model, om, prompt = mini
    G = 4
    greedy = om.greedy(prompt, 40)
    plans = []

    def drafts_for(emitted, kind):
        n = len(emitted)
        d = list(greedy[n:n + G])
        if kind == 1:
            d[2] = (d[2] + 1) % model.info.vocab
        if kind == 2:
            d[0] = (d[0] + 1) % model.info.vocab
        return d

    kinds = [0, 1, 2, 0, 1]
    st = _state(model)
    emitted = [st.prefill(prompt)]
    for k in kinds:
        d = drafts_for(emitted, k)
        plans.append(d)
        st.spec_step(G, d)
        toks, pos, acc, _ = st.read()
        emitted = list(toks)
        assert acc == {0: G, 1: 2, 2: 0}[k]
    assert emitted == greedy[:len(emitted)]
    out_o, ref = om.spec_decode(prompt, len(kinds), G, drafts=lambda s: plans[s])
    assert emitted == out_o
    lg, _, _ = st.last_verify()
    assert O.norm_rel(lg, ref[-1]["logits"]).max() < LOGIT_TOL


def test_gamma_zero_is_greedy(O, mini):
    model, om, prompt = mini
    st = _state(model)
    st.prefill(prompt)
    for _ in range(15):
        st.spec_step(0)
    toks, pos, acc, _ = st.read()
    assert list(toks) == om.greedy(prompt, 16)
    assert pos == len(prompt) + 15


def test_state_reset_and_errors(pkg, mini):
    model, om, prompt = mini
    st = _state(model, 64)
    a = st.prefill(prompt)
    st.reset()
    b = st.prefill(prompt)
    assert a == b
    with pytest.raises(pkg.IfrError, match="gamma"):
        st.spec_step(9)
    with pytest.raises(pkg.IfrError, match="out of range"):
        st.spec_step(2, [0, model.info.vocab])
    with pytest.raises(pkg.IfrError, match="max_ctx"):
        st.prefill(np.zeros(60, np.int32))


def test_config1_tiny_model_matches_oracle(O, pkg, ctx):
    """BASELINE config 1 shapes (tiny Qwen3.5 hybrid, Q4_K / Q6_K, 128-token
    prompt): prefill + two MTP spec steps, logits and tokens vs the oracle"""
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model, State
    path = synth.cached("tiny", seed=0)
    model = Model(ctx, path)
    om = O.OracleModel(gguf.GGUFFile(path), 300)
    prompt = synth.prompt(model.info.vocab, 128, seed=0)
    st = State(model, 300)
    first = st.prefill(prompt)
    out_o, ref = om.spec_decode(prompt, 2, 4)
    assert first == out_o[0]
    for s in range(2):
        st.spec_step(4)
        lg, _, tk = st.last_verify()
        assert list(tk[1:]) == ref[s]["drafts"]
        assert O.norm_rel(lg, ref[s]["logits"]).max() < LOGIT_TOL
    toks, *_ = st.read()
    assert list(toks) == out_o
    del om


def test_step_in_parts_matches_fused_step(mini):
    """ifr_draft_mtp + ifr_verify_step + the caller's greedy acceptance (host
    argmax of the returned logits) + ifr_rollback reproduce ifr_spec_step:
    same drafts, logits, emitted tokens and positions"""
    import torch
    model, om, prompt = mini
    G, steps = 4, 5
    a, b = _state(model), _state(model)
    a.prefill(prompt)
    b.prefill(prompt)
    V = model.info.vocab
    lg = torch.empty((G + 1) * V, dtype=torch.float32, device="cuda")
    for s in range(steps):
        a.spec_step(G)
        la, _, ta = a.last_verify()
        d = b.draft_mtp(G)
        b.verify_step(G, None, lg)
        lb = lg.view(G + 1, V).cpu().numpy()
        assert list(d[0]) == list(ta[1:]), (s, d, ta)
        assert np.array_equal(lb, la), s
        am = lb.argmax(axis=1)
        acc = 0
        while acc < G and am[acc] == d[0][acc]:
            acc += 1
        toks = np.full(G + 1, -1, np.int32)
        toks[:acc] = d[0][:acc]
        toks[acc] = am[acc]
        b.rollback([acc], toks[None])
        ra, rb = a.read(), b.read()
        assert list(ra[0]) == list(rb[0]) and ra[1:] == rb[1:], (s, ra, rb)


def test_step_in_parts_forced_and_errors(mini):
    """caller-chosen drafts and acceptance: a rejection at the first draft with
    a token of the caller's choice, then the fused step continues from it;
    out-of-order calls are rejected"""
    from inferno_b200._lib import IfrError
    model, om, prompt = mini
    G = 3
    st = _state(model)
    g0 = st.prefill(prompt)
    n0, pos0 = len(st.read()[0]), st.read()[1]
    st.verify_step(G, np.array([[1, 2, 3]], np.int32))
    with pytest.raises(IfrError):
        st.verify_step(G, np.array([[1, 2, 3]], np.int32))
    with pytest.raises(IfrError):
        st.spec_step(G)
    with pytest.raises(IfrError):
        st.rollback([G + 1], np.zeros((1, G + 1), np.int32))
    st.rollback([0], np.array([[77, -1, -1, -1]], np.int32))
    toks, pos, acc, _ = st.read()
    assert len(toks) == n0 + 1 and toks[-1] == 77 and pos == pos0 + 1 and acc == 0
    with pytest.raises(IfrError):
        st.rollback([0], np.array([[77, -1, -1, -1]], np.int32))
    # the sequence is now prompt, g0, 77: the next fused step's first emitted
    # token is the greedy successor of that (a fresh state's prefill)
    ref = _state(model)
    first = ref.prefill(np.concatenate([np.asarray(prompt, np.int32), np.array([g0, 77], np.int32)]))
    st.spec_step(G)
    assert st.read()[0][n0 + 1] == first


def test_config1_128_greedy_tokens_every_step(O, pkg, ctx):
    """BASELINE config 1 end to end: the seeded tiny model, 128-token prompt,
    128 greedy tokens by speculative decoding (gamma 4).  Random weights make
    the MTP drafts miss, so the drafts are forced from the oracle's greedy
    continuation in a repeating plan - all accepted, a wrong third draft, a
    wrong first draft - which runs the full-accept and partial-accept
    rollbacks (SSM replay record, conv history, KV overwrite) at config-1
    shapes.  Every step: verify logits within 1e-4 of the oracle, accept
    counts and emitted tokens equal; the 128 tokens equal plain greedy."""
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model, State
    path = synth.cached("tiny", seed=0)
    model = Model(ctx, path)
    V = model.info.vocab
    om = O.OracleModel(gguf.GGUFFile(path), 300)
    prompt = synth.prompt(V, 128, seed=0)
    n_gen, G = 128, 4
    greedy = om.greedy(list(prompt), n_gen + G + 1)
    st = State(model, 300)
    emitted = [int(st.prefill(prompt))]
    plans, kinds, accs, logits = [], [0, 1, 0, 2], [], []
    while len(emitted) < n_gen:
        k = kinds[len(plans) % len(kinds)]
        d = list(greedy[len(emitted):len(emitted) + G])
        if k == 1:
            d[2] = (d[2] + 1) % V
        elif k == 2:
            d[0] = (d[0] + 1) % V
        plans.append(d)
        st.spec_step(G, d)
        logits.append(st.last_verify()[0])
        toks, pos, acc, _ = st.read()
        accs.append(acc)
        assert acc == {0: G, 1: 2, 2: 0}[k], (len(plans), acc)
        emitted = [int(t) for t in toks]
    assert emitted[:n_gen] == greedy[:n_gen]
    out, ref = om.spec_decode(list(prompt), len(plans), G, drafts=lambda s: plans[s])
    assert emitted == out
    for s, r in enumerate(ref):
        assert r["acc"] == accs[s], s
        assert O.norm_rel(logits[s], r["logits"]).max() < LOGIT_TOL, s
    st.free()
    model.free()
    om.close()
