"""GPU parity of the chunked prefill of one request (forward_cpu! over the
prompt, reference src/ModelCPU.jl:1325): the prompt goes through the model in
chunks of 64 tokens - every projection over the chunk's 64 columns, the
GatedDeltaNet layers scanning the chunk inside one launch and committing its
state at once (no replay record), attention in 8-token sub-calls at their
positions.  Checked against the oracle's token-by-token forward: the first
token, the final hidden state and the logits after the prompt, and the spec
steps that continue from the committed state.

  * default, exact path (every projection on the exact small-N kernel, in
    passes of 8 columns over the chunk): 1e-4;
  * ifr_ctx_set_prefill_dense (the chunk's projections on the dense tcgen05
    GEMM, fp16 operands): 1e-2, the north star's bound for reduced-precision
    accumulation.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-4
DENSE_TOL = 1e-2


def _oracle_prefill(om, prompt):
    om.reset()
    for i, t in enumerate(prompt):
        lg, hd = om.forward_token(int(t), i)
    return lg, hd


def _check_prefill(O, ctx, path, P, max_ctx, seed, exact, steps=2, G=4):
    from inferno_b200 import synth, gguf
    from inferno_b200.engine import Model, State
    model = Model(ctx, path)
    om = O.OracleModel(gguf.GGUFFile(path), max_ctx)
    prompt = synth.prompt(model.info.vocab, P, seed=seed)
    if not exact:
        ctx.set_prefill_dense(True)
    try:
        st = State(model, max_ctx)
        first = int(st.prefill(prompt))
        lg_o, hd_o = _oracle_prefill(om, prompt)
        # the last prompt token's column: its hidden and logits
        _, hid, toks = st.last_verify()
        tol = LOGIT_TOL if exact else DENSE_TOL
        assert O.norm_rel(hid.reshape(1, -1), hd_o.reshape(1, -1)).max() < tol
        if exact:
            assert first == int(np.argmax(lg_o))
        pos = st.read()[1]
        assert pos == P
        # continue with spec steps from the committed state
        if exact:
            out, ref = om.spec_decode(list(prompt), steps, G)
            for s in range(steps):
                st.spec_step(G)
                lg, _, tk = st.last_verify()
                assert list(tk[1:]) == ref[s]["drafts"], s
                assert O.norm_rel(lg, ref[s]["logits"]).max() < LOGIT_TOL, s
            assert [int(t) for t in st.read()[0]] == out
        st.free()
    finally:
        ctx.set_prefill_dense(False)
        om.close()
        model.free()


@pytest.mark.parametrize("P", [2048, 200, 70])
def test_chunked_prefill_mini_exact(O, ctx, P):
    """the small hybrid (SSM head dim 64), up to a 2048-token prompt (32 chunks
    of 64 and the last token), exact path"""
    from inferno_b200 import synth
    _check_prefill(O, ctx, synth.cached("mini", seed=1), P, P + 64, seed=P, exact=True)


def test_chunked_prefill_config1_shapes_exact(O, ctx):
    """config 1's shapes (SSM head dim 128, attention head dim 256, 24 layers),
    a 200-token prompt: three chunks of 64, a chunk of 7, the last token"""
    from inferno_b200 import synth
    _check_prefill(O, ctx, synth.cached("tiny", seed=0), 200, 300, seed=5, exact=True, steps=1)


def test_chunked_prefill_dense_path(O, ctx):
    """opt-in: the chunk's projections on the dense tcgen05 GEMM"""
    from inferno_b200 import synth
    _check_prefill(O, ctx, synth.cached("mini", seed=1), 1500, 1600, seed=3, exact=False)


def test_chunked_prefill_gemma_blocks(O, ctx):
    """attention-only Gemma4 blocks: sliding windows across chunk borders"""
    from inferno_b200 import synth
    _check_prefill(O, ctx, synth.cached("gemma_mini", seed=1), 150, 256, seed=8, exact=True, steps=0)
