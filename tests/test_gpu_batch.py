"""GPU parity of the batched engine (ifr_state_create_batch: several requests
advancing together) against the CPU oracle run on each request's prompt alone,
through the C ABI.

  * exact path (every projection on the small-N kernel): the same bar as the
    one-request engine - drafts, accept counts and emitted tokens equal,
    verify logits within LOGIT_TOL;
  * dense path (projections of many columns on the tcgen05 kernel, fp16
    operands): verify logits within DENSE_TOL of the oracle, the north star's
    bound for reduced-precision accumulation, with forced drafts so both sides
    see the same tokens.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4   # exact path, f32 accumulation on both sides
DENSE_TOL = 1e-2   # dense path: fp16 operands, f32 accumulation
# bf16 caches: both sides round every cached row to bf16, but a row value whose
# f32 differs by ~1e-7 between the two (the norm's summation order) can round
# to the neighbouring bf16 value, 2^-8 relative away; a few such flips over a
# few hundred thousand cached values move the logits by ~1e-4
KV16_TOL = 1e-3


@pytest.fixture(scope="module")
def mini(pkg, O, ctx):
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model
    path = synth.cached("mini", seed=1)
    model = Model(ctx, path)
    om = O.OracleModel(gguf.GGUFFile(path), 512)
    return model, om


def _prompts(vocab, B, n):
    from inferno_b200 import synth
    return np.stack([synth.prompt(vocab, n, seed=100 + b) for b in range(B)])


@pytest.mark.parametrize("B,G,dense_min", [(2, 3, None), (3, 4, 10**6), (5, 2, 10**6)])
def test_batch_exact_matches_oracle(O, ctx, mini, B, G, dense_min):
    from inferno_b200.engine import State
    model, om = mini
    V = model.info.vocab
    steps = 5
    prompts = _prompts(V, B, 21)
    ref = [om.spec_decode(list(p), steps, G) for p in prompts]
    if dense_min:
        ctx.set_dense_min_cols(dense_min)
    try:
        st = State(model, 512, batch=B)
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
                _, pos, acc, nst = st.read(b)
                assert acc == r["acc"] and nst == s + 1 and pos == r["pos"] + acc + 1, (b, s)
        for b in range(B):
            toks, *_ = st.read(b)
            assert list(toks) == ref[b][0], b
        st.free()
    finally:
        ctx.set_dense_min_cols(24)


def test_batch_dense_logits_within_tolerance(O, ctx, mini):
    """prefill (B x 8 columns per chunk) and a verify of B x 5 columns on the
    dense tensor-core path; drafts forced to the oracle's greedy continuation"""
    from inferno_b200.engine import State
    model, om = mini
    V = model.info.vocab
    B, G = 6, 4
    prompts = _prompts(V, B, 30)
    greedy = [om.greedy(list(p), G + 2) for p in prompts]
    ctx.set_dense_min_cols(8)
    try:
        st = State(model, 512, batch=B)
        firsts = st.prefill(prompts)
        assert [int(f) for f in firsts] == [g[0] for g in greedy]
        drafts = np.array([g[1:G + 1] for g in greedy], np.int32)
        st.spec_step(G, drafts)
        lg, _, tk = st.last_verify()
        lg = lg.reshape(B, G + 1, V)
        for b, p in enumerate(prompts):
            # oracle logits of the same columns: prompt, then [first, drafts]
            om.reset()
            for i, t in enumerate(p):
                om.forward_token(int(t), i)
            cols = greedy[b][:G + 1]
            ref = np.stack([om.forward_token(t, len(p) + j)[0] for j, t in enumerate(cols)])
            assert list(tk.reshape(B, G + 1)[b]) == cols
            err = O.norm_rel(lg[b], ref)
            assert err.max() < DENSE_TOL, (b, err)
        _, pos, acc, _ = st.read(0)
        assert acc == G  # the forced drafts are the greedy continuation
        st.free()
    finally:
        ctx.set_dense_min_cols(24)


def test_batch_argument_errors(pkg, mini):
    from inferno_b200._lib import load
    import ctypes
    model, _ = mini
    h = ctypes.c_void_p()
    assert load().ifr_state_create_batch(model.handle, 512, 0, ctypes.byref(h)) != 0
    assert load().ifr_state_create_batch(model.handle, 512, 10**6, ctypes.byref(h)) != 0


@pytest.mark.parametrize("B,P,max_ctx", [(1, 300, 1024), (3, 200, 512)])
def test_split_kv_attention_matches_oracle(O, ctx, mini, B, P, max_ctx):
    """split-KV attention (one request with a long cache, or a batch): the
    keys of every request spread over several slices whose partial softmax
    states are merged; the exact-path bar (tokens equal, logits 1e-4)"""
    from inferno_b200.engine import State
    model, om = mini
    V = model.info.vocab
    G, steps = 4, 3
    prompts = _prompts(V, B, P)
    ref = [om.spec_decode(list(p), steps, G) for p in prompts]
    ctx.set_dense_min_cols(10**6)  # every projection on the exact small-N kernel
    try:
        st = State(model, max_ctx, batch=B)
        firsts = st.prefill(prompts if B > 1 else prompts[0])
        firsts = np.atleast_1d(firsts)
        assert [int(f) for f in firsts] == [r[0][0] for r in ref]
        for s in range(steps):
            st.spec_step(G)
            lg, _, tk = st.last_verify()
            lg = lg.reshape(B, G + 1, V)
            tk = tk.reshape(B, G + 1)
            for b in range(B):
                r = ref[b][1][s]
                assert list(tk[b, 1:]) == r["drafts"], (b, s)
                assert O.norm_rel(lg[b], r["logits"]).max() < LOGIT_TOL, (b, s)
        for b in range(B):
            toks, *_ = st.read(b)
            assert list(toks) == ref[b][0], b
        st.free()
    finally:
        ctx.set_dense_min_cols(24)


def test_batch_dense_fp16_stages_bit_exact(pkg, ctx):
    """ifr_ctx_set_dense_f16_weights: a batched state whose model keeps fp16
    operand stages of every projection gives bit-for-bit the logits and
    tokens of one whose dense GEMMs dequantize on the fly"""
    from inferno_b200 import synth
    from inferno_b200.engine import Model, State
    path = synth.cached("mini", seed=1)
    out = []
    for f16 in (False, True):
        ctx.set_dense_f16_weights(f16)
        ctx.set_dense_min_cols(8)
        model = Model(ctx, path)
        try:
            B, G = 6, 4
            prompts = _prompts(model.info.vocab, B, 30)
            st = State(model, 256, batch=B)
            st.prefill(prompts)
            for _ in range(2):
                st.spec_step(G)
            lg, _, tk = st.last_verify()
            out.append((lg.copy(), tk.copy(), [list(st.read(b)[0]) for b in range(B)]))
            st.free()
        finally:
            ctx.set_dense_min_cols(24)
            ctx.set_dense_f16_weights(True)
            model.free()
    (l0, t0, e0), (l1, t1, e1) = out
    assert np.array_equal(l0.view(np.uint32), l1.view(np.uint32))
    assert list(t0) == list(t1) and e0 == e1


def _kv_bf16_run(O, ctx, model, om, B, P, max_ctx, G=4, steps=3):
    """spec steps of a state with bf16 attention caches against the oracle
    rounding its cache rows the same way (or_model_set_kv_bf16): drafts,
    tokens and accept counts equal, verify logits within KV16_TOL; the first
    verify's logits also within DENSE_TOL (1e-2) of the f32-cache oracle"""
    from inferno_b200.engine import State
    V = model.info.vocab
    prompts = _prompts(V, B, P)
    om.set_kv_bf16(True)
    try:
        ref = [om.spec_decode(list(p), steps, G) for p in prompts]
    finally:
        om.set_kv_bf16(False)
    # the f32-cache oracle's first verify (same drafts: the bf16 cache enters
    # only through the attention), for the north star's 1e-2 bound
    ref32 = [om.spec_decode(list(p), 1, G, drafts=lambda s, b=b: ref[b][1][0]["drafts"])[1][0]["logits"]
             for b, p in enumerate(prompts)]
    ctx.set_dense_min_cols(10**6)  # every projection on the exact small-N kernel
    ctx.set_kv_bf16(True)
    try:
        st = State(model, max_ctx, batch=B)
        firsts = np.atleast_1d(st.prefill(prompts if B > 1 else prompts[0]))
        assert [int(f) for f in firsts] == [r[0][0] for r in ref]
        for s in range(steps):
            st.spec_step(G)
            lg, _, tk = st.last_verify()
            lg = lg.reshape(B, G + 1, V)
            tk = tk.reshape(B, G + 1)
            for b in range(B):
                r = ref[b][1][s]
                assert list(tk[b, 1:]) == r["drafts"], (b, s)
                assert O.norm_rel(lg[b], r["logits"]).max() < KV16_TOL, (b, s)
                if s == 0:
                    assert O.norm_rel(lg[b], ref32[b]).max() < DENSE_TOL, b
        for b in range(B):
            toks, *_ = st.read(b)
            assert list(toks) == ref[b][0], b
        st.free()
    finally:
        ctx.set_kv_bf16(False)
        ctx.set_dense_min_cols(24)


@pytest.mark.parametrize("B,P,max_ctx", [(3, 200, 512), (1, 300, 1024)])
def test_kv_bf16_head_dim_64(O, ctx, mini, B, P, max_ctx):
    """ifr_ctx_set_kv_bf16 on the mini model (head dim 64, 2 q heads per KV
    head): a batch, and one request whose long cache takes the split path"""
    model, om = mini
    _kv_bf16_run(O, ctx, model, om, B, P, max_ctx)


def test_kv_bf16_head_dim_256(O, pkg, ctx):
    """ifr_ctx_set_kv_bf16 at config-1/4 attention shapes (head dim 256, 4 q
    heads per KV head: 20 rows of 5 verify columns in two m-tiles)"""
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model
    path = synth.cached("tiny", seed=0)
    model = Model(ctx, path)
    om = O.OracleModel(gguf.GGUFFile(path), 256)
    try:
        _kv_bf16_run(O, ctx, model, om, 2, 90, 256, steps=2)
    finally:
        om.close()
        model.free()


def test_kv_bf16_not_on_short_single_request(ctx, mini):
    """one request with a short cache keeps the single-launch f32 attention
    (the flag applies to split-KV states only): identical to the flag off"""
    from inferno_b200.engine import State
    model, _ = mini
    prompt = _prompts(model.info.vocab, 1, 40)[0]
    outs = []
    for on in (False, True):
        ctx.set_kv_bf16(on)
        try:
            st = State(model, 256)
            st.prefill(prompt)
            for _ in range(3):
                st.spec_step(4)
            outs.append(st.last_verify()[0].copy())
            st.free()
        finally:
            ctx.set_kv_bf16(False)
    assert np.array_equal(outs[0], outs[1])
