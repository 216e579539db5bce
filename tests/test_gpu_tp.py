"""GPU parity of the tensor-parallel model (ifr_model_load_gguf_tp): every rank
holds a shard of the attention heads, FFN units and lm_head rows, the residual
is summed over the ranks after the row-parallel projections, and greedy
acceptance takes the argmax over all vocabulary shards.

  * one rank (no NCCL needed): the tensor-parallel path must give exactly the
    plain engine's logits and tokens, and match the oracle;
  * two ranks (needs 2 GPUs and NCCL; skipped otherwise): spawned processes,
    one per GPU; the concatenated logits shards and the emitted tokens match
    the oracle.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4


@pytest.fixture(scope="module")
def tpm(pkg, O, ctx):
    from inferno_b200 import synth, gguf
    path = synth.cached("tp_mini", seed=1)
    om = O.OracleModel(gguf.GGUFFile(path), 512)
    return path, om


def _plan(om, prompt, G, steps):
    """forced drafts: the greedy continuation with one wrong draft in every
    other step (full accept, then partial), and the oracle's reference run"""
    greedy = om.greedy(list(prompt), 64)

    def drafts(s, emitted):
        d = list(greedy[len(emitted):len(emitted) + G])
        if s % 2:
            d[1] = (d[1] + 7) % om.vocab
        return d
    return greedy, drafts


def _run(model_ctx, path, comm, prompt, G, steps, om):
    from inferno_b200.engine import Model, State
    model = Model(model_ctx, path, comm)
    st = State(model, 256)
    emitted = [int(st.prefill(prompt))]
    greedy, drafts = _plan(om, prompt, G, steps)
    logits, used = [], []
    for s in range(steps):
        d = drafts(s, emitted)
        used.append(d)
        st.spec_step(G, d)
        lg, _, _ = st.last_verify()
        logits.append(lg)
        emitted = [int(t) for t in st.read()[0]]
    st.free()
    model.free()
    return emitted, logits, used


def test_tp_single_rank_equals_plain_and_oracle(O, pkg, ctx, tpm):
    from inferno_b200.engine import Comm
    from inferno_b200 import synth
    path, om = tpm
    prompt = synth.prompt(om.vocab, 20, seed=3)
    G, steps = 3, 4
    comm = Comm(ctx, 0, 1)
    try:
        e_tp, l_tp, used = _run(ctx, path, comm, prompt, G, steps, om)
    finally:
        comm.free()
    e_pl, l_pl, _ = _run(ctx, path, None, prompt, G, steps, om)
    assert e_tp == e_pl
    for a, b in zip(l_tp, l_pl):
        assert np.array_equal(a, b)
    out, ref = om.spec_decode(list(prompt), steps, G, drafts=lambda s: used[s])
    assert e_tp == out
    for s in range(steps):
        assert O.norm_rel(l_tp[s], ref[s]["logits"]).max() < LOGIT_TOL


def _rank_main(rank, world, uid, path, prompt, G, steps, drafts_all, q):
    import os
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch
    import __graft_entry__ as ge
    pkg = ge.load_package()
    pkg.load()
    from inferno_b200.engine import Comm, Model, State
    torch.cuda.set_device(rank)
    ctx = pkg.Context(rank)
    comm = Comm(ctx, rank, world, uid)
    model = Model(ctx, path, comm)
    st = State(model, 256)
    st.prefill(prompt)
    logits = []
    for s in range(steps):
        st.spec_step(G, drafts_all[s])
        lg, _, _ = st.last_verify()
        logits.append(lg)
    toks = [int(t) for t in st.read()[0]]
    st.free()
    model.free()
    comm.free()
    ctx.close()
    q.put((rank, toks, logits))


@pytest.mark.parametrize("preset", ["tp_mini", "gemma_narrow"])
def test_tp_two_ranks_match_oracle(O, preset):
    """tp_mini, and gemma_narrow: the Gemma4-shape target's widths (hidden
    5376, 32 q / 16 kv x 128, FFN 21504 = 84 units split 42/42) with 2 layers"""
    import torch
    import torch.multiprocessing as mp
    from inferno_b200.engine import Comm
    from inferno_b200 import synth, gguf
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if not Comm.available():
        pytest.skip("NCCL not available")
    path = synth.cached(preset, seed=1)
    om = O.OracleModel(gguf.GGUFFile(path), 512)
    prompt = synth.prompt(om.vocab, 20, seed=4)
    G, steps = 3, 4
    greedy = om.greedy(list(prompt), 64)
    # a fixed draft plan that the oracle and both ranks replay
    used = [_fixed(greedy, s, G, om.vocab) for s in range(steps)]
    out, ref = om.spec_decode(list(prompt), steps, G, drafts=lambda s: used[s])
    uid = Comm.unique_id()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    procs = [mpc.Process(target=_rank_main, args=(r, 2, uid, path, prompt, G, steps, used, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, toks, lg = q.get(timeout=300)
        res[r] = (toks, lg)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0][0] == out and res[1][0] == out
    for s in range(steps):
        full = np.concatenate([res[0][1][s], res[1][1][s]], axis=1)
        assert O.norm_rel(full, ref[s]["logits"]).max() < LOGIT_TOL, s
    om.close()


def _fixed(greedy, s, G, vocab):
    """step s's drafts for the two-rank test: the greedy tokens from offset
    1 + s (a fixed plan that both the oracle and the ranks replay)"""
    d = [int(t) for t in greedy[1 + s:1 + s + G]]
    if s % 2:
        d[1] = (d[1] + 7) % vocab
    return d


def test_draft_model_spec_decode_matches_oracle(O, pkg, ctx, tpm):
    """ifr_spec_step_draft: a second (attention-only) model drafts greedily,
    the target verifies; tokens and verify logits vs the oracle running the
    same protocol with both models"""
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model, State
    path, om = tpm
    dpath = synth.cached("tp_mini", seed=2)
    dm = O.OracleModel(gguf.GGUFFile(dpath), 512)
    prompt = [int(t) for t in synth.prompt(om.vocab, 18, seed=5)]
    G, steps = 3, 4
    target, draft = Model(ctx, path), Model(ctx, dpath)
    ts, ds = State(target, 256), State(draft, 256)
    first = int(ts.prefill(np.array(prompt, np.int32)))
    ds.prefill(np.array(prompt, np.int32))
    plan = []

    def drafts_at(out):
        # the draft model's greedy continuation of prompt + emitted tokens
        return [int(t) for t in dm.greedy(prompt + out, G)]
    out = [first]
    for s in range(steps):
        plan.append(drafts_at(out))
        out, _ = om.spec_decode(prompt, s + 1, G, drafts=lambda i: plan[i])
    ref_out, ref = om.spec_decode(prompt, steps, G, drafts=lambda i: plan[i])
    for s in range(steps):
        ts.spec_step_draft(ds, G)
        lg, _, tk = ts.last_verify()
        assert list(tk[1:]) == plan[s], (s, tk, plan[s])
        assert O.norm_rel(lg, ref[s]["logits"]).max() < LOGIT_TOL, s
    toks, pos, acc, nst = ts.read()
    assert [int(t) for t in toks] == ref_out
    ts.free()
    ds.free()
