"""GPU parity at the large configurations' widths, with few layers so that the
CPU oracle can follow: the kernel instantiations that config 4 (the ~9B-shape
hybrid, batched requests) and config 5 (the Gemma4-shape target, tensor
parallel) run, which the small test models do not reach.

  * 9b_narrow (hidden 4096, 16 q / 4 kv heads x 256, 32 SSM heads x 128, FFN
    12288, Q6_K ffn_down, vocab 151936; 3 SSM layers + 1 attention layer):
    the batched GatedDeltaNet kernel at head dim 128 and split-KV attention at
    head dim 256, on 4 requests on the exact path (logits within 1e-4, tokens
    equal) and on 64 requests on the dense tensor-core path (logits within
    1e-2 for the requests checked against the oracle);
  * gemma_narrow (hidden 5376, 32 q / 16 kv x 128, FFN 21504; 2 layers,
    vocab 32768): the tensor-parallel engine on one rank equals the plain
    engine and the oracle (1e-4).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4   # exact path, f32 accumulation on both sides
DENSE_TOL = 1e-2   # dense path: fp16 operands, f32 accumulation


@pytest.fixture(scope="module")
def narrow9b(pkg, O, ctx):
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model
    path = synth.cached("9b_narrow", seed=2)
    model = Model(ctx, path)
    om = O.OracleModel(gguf.GGUFFile(path), 160)
    yield model, om
    om.close()
    model.free()


def _prompts(vocab, B, n, seed):
    from inferno_b200 import synth
    return np.stack([synth.prompt(vocab, n, seed=seed + b) for b in range(B)])


def test_9b_widths_batch_exact_matches_oracle(O, ctx, narrow9b):
    """4 requests, MTP drafts, exact activations on every projection"""
    from inferno_b200.engine import State
    model, om = narrow9b
    i = model.info
    assert (i.hidden, i.n_head, i.n_kv_head, i.head_dim, i.ssm_heads, i.ssm_head_dim, i.ffn) == \
        (4096, 16, 4, 256, 32, 128, 12288)
    B, G, steps = 4, 4, 2
    V = i.vocab
    prompts = _prompts(V, B, 12, 500)
    ref = [om.spec_decode(list(p), steps, G) for p in prompts]
    ctx.set_dense_min_cols(10**6)
    try:
        st = State(model, 160, batch=B)
        firsts = st.prefill(prompts)
        assert [int(f) for f in firsts] == [r[0][0] for r in ref]
        for s in range(steps):
            st.spec_step(G)
            lg, hd, tk = st.last_verify()
            lg = lg.reshape(B, G + 1, V)
            hd = hd.reshape(B, G + 1, -1)
            tk = tk.reshape(B, G + 1)
            for b in range(B):
                r = ref[b][1][s]
                assert list(tk[b, 1:]) == r["drafts"], (b, s)
                assert O.norm_rel(lg[b], r["logits"]).max() < LOGIT_TOL, (b, s)
                assert O.norm_rel(hd[b], r["hidden"]).max() < LOGIT_TOL, (b, s)
        for b in range(B):
            assert list(st.read(b)[0]) == ref[b][0], b
        st.free()
    finally:
        ctx.set_dense_min_cols(24)


def test_9b_widths_batch64_dense_within_tolerance(O, ctx, narrow9b):
    """64 requests (config 4's batch on one GPU): prefill (64 x 8 columns)
    and one verify of 64 x 5 columns on the dense tcgen05 path; four requests
    spread over the batch are checked against the oracle with drafts forced
    to their greedy continuation (the others get arbitrary drafts)"""
    from inferno_b200.engine import State
    model, om = narrow9b
    V = model.info.vocab
    B, G, P = 64, 4, 8
    prompts = _prompts(V, B, P, 900)
    checked = [0, 21, 42, 63]
    greedy = {b: om.greedy(list(prompts[b]), G + 2) for b in checked}
    rng = np.random.default_rng(64)
    drafts = rng.integers(0, V, (B, G)).astype(np.int32)
    for b in checked:
        drafts[b] = greedy[b][1:G + 1]
    st = State(model, 64, batch=B)
    firsts = st.prefill(prompts)
    for b in checked:
        assert int(firsts[b]) == greedy[b][0], b
    st.spec_step(G, drafts)
    lg, _, tk = st.last_verify()
    lg = lg.reshape(B, G + 1, V)
    tk = tk.reshape(B, G + 1)
    for b in checked:
        om.reset()
        for j, t in enumerate(prompts[b]):
            om.forward_token(int(t), j)
        cols = greedy[b][:G + 1]
        ref = np.stack([om.forward_token(t, P + j)[0] for j, t in enumerate(cols)])
        assert list(tk[b]) == cols
        err = O.norm_rel(lg[b], ref)
        assert err.max() < DENSE_TOL, (b, err)
        assert st.read(b)[2] == G  # the forced drafts are the greedy continuation
    st.free()


def test_gemma_widths_tensor_parallel_single_rank(O, pkg, ctx):
    """the tensor-parallel engine on one rank at the Gemma4-shape target's
    widths: identical to the plain engine, and within 1e-4 of the oracle,
    with forced drafts (full accept, then a wrong second draft)"""
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Comm, Model, State
    path = synth.cached("gemma_narrow", seed=3)
    om = O.OracleModel(gguf.GGUFFile(path), 96)
    prompt = synth.prompt(om.vocab, 10, seed=7)
    G, steps = 3, 3
    greedy = om.greedy(list(prompt), 32)

    def run(comm):
        model = Model(ctx, path, comm)
        i = model.info
        assert (i.hidden, i.n_head, i.n_kv_head, i.head_dim, i.ffn) == (5376, 32, 16, 128, 21504)
        st = State(model, 96)
        emitted = [int(st.prefill(prompt))]
        logits, used = [], []
        for s in range(steps):
            d = list(greedy[len(emitted):len(emitted) + G])
            if s % 2:
                d[1] = (d[1] + 7) % om.vocab
            used.append(d)
            st.spec_step(G, d)
            logits.append(st.last_verify()[0])
            emitted = [int(t) for t in st.read()[0]]
        st.free()
        model.free()
        return emitted, logits, used

    comm = Comm(ctx, 0, 1)
    try:
        e_tp, l_tp, used = run(comm)
    finally:
        comm.free()
    e_pl, l_pl, _ = run(None)
    assert e_tp == e_pl
    for a, b in zip(l_tp, l_pl):
        assert np.array_equal(a, b)
    out, ref = om.spec_decode(list(prompt), steps, G, drafts=lambda s: used[s])
    assert e_tp == out
    for s in range(steps):
        assert O.norm_rel(l_tp[s], ref[s]["logits"]).max() < LOGIT_TOL, s
    om.close()
