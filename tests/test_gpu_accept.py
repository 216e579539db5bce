"""GPU parity of the acceptance kernels: accept counts, emitted tokens and
drawn drafts bit-exact with the CPU oracle for the same supplied uniforms."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _case(rng, B, G, V, noise=1.0, scale=3.0):
    tgt = rng.normal(0, scale, (B, G + 1, V)).astype(np.float32)
    dft = (tgt[:, :G] + rng.normal(0, noise, (B, G, V))).astype(np.float32)
    u = rng.random((B, 2 * G + 1), dtype=np.float32)
    return tgt, dft, u


def _run(ctx, tgt, dft, u, T, dtok=None):
    import torch
    d = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    acc, out, dout = ctx.accept(d(tgt), d(dft), d(u), T, d(dtok))
    return acc.cpu().numpy(), out.cpu().numpy(), dout.cpu().numpy()


@pytest.mark.parametrize("B,G,V", [(4, 3, 5000), (3, 5, 3001), (2, 1, 7), (16, 4, 2048)])
def test_accept_bit_exact(O, ctx, B, G, V):
    rng = np.random.default_rng(B * 100 + G * 10 + V)
    for noise in (0.3, 1.0, 3.0):
        tgt, dft, u = _case(rng, B, G, V, noise)
        got = _run(ctx, tgt, dft, u, 0.8)
        ref = O.accept(tgt, dft, u, 0.8)
        for g, r, name in zip(got, ref, ("accept_count", "out_tokens", "draft_tokens")):
            assert np.array_equal(g, r), (name, noise, g, r)


def test_accept_config3_shape_subset(O, ctx):
    """vocab 151936, draft length 5, temperature 0.8, 4 sequences"""
    rng = np.random.default_rng(33)
    tgt, dft, u = _case(rng, 4, 5, 151936)
    got = _run(ctx, tgt, dft, u, 0.8)
    ref = O.accept(tgt, dft, u, 0.8)
    for g, r in zip(got, ref):
        assert np.array_equal(g, r)


def test_accept_config3_full_batch(O, ctx):
    """BASELINE config 3 at its stated shape: 64 sequences x draft length 5,
    vocab 151936, target ~N(0, 3), draft = target + N(0, 1), T = 0.8,
    supplied seeded uniforms; accept counts, emitted and drawn tokens
    bit-exact"""
    rng = np.random.default_rng(3)
    tgt, dft, u = _case(rng, 64, 5, 151936)
    got = _run(ctx, tgt, dft, u, 0.8)
    ref = O.accept(tgt, dft, u, 0.8)
    for g, r, name in zip(got, ref, ("accept_count", "out_tokens", "draft_tokens")):
        assert np.array_equal(g, r), name
    assert 0 < ref[0].mean() < 5  # a mix of acceptances, not a degenerate case


def test_accept_given_drafts(O, ctx):
    rng = np.random.default_rng(34)
    B, G, V = 6, 4, 4000
    tgt, dft, u = _case(rng, B, G, V)
    dtok = rng.integers(0, V, (B, G)).astype(np.int32)
    dtok[0] = np.argmax(dft[0], axis=-1)
    got = _run(ctx, tgt, dft, u, 1.3, dtok)
    ref = O.accept(tgt, dft, u, 1.3, dtok)
    for g, r in zip(got, ref):
        assert np.array_equal(g, r)


def test_accept_identical_rows_zero_residual(O, ctx):
    """draft == target: every ratio is 1, all accepted; forcing u_a = 1
    rejects and exercises the zero-residual fallback"""
    rng = np.random.default_rng(35)
    B, G, V = 3, 3, 3000
    tgt = rng.normal(0, 3, (B, G + 1, V)).astype(np.float32)
    dft = tgt[:, :G].copy()
    u = rng.random((B, 2 * G + 1), dtype=np.float32) * 0.99
    got = _run(ctx, tgt, dft, u, 0.8)
    assert (got[0] == G).all()
    u[:, G] = 1.0  # u_a[0] = 1 -> rejected at 0 with residual 0
    got = _run(ctx, tgt, dft, u, 0.8)
    ref = O.accept(tgt, dft, u, 0.8)
    for g, r in zip(got, ref):
        assert np.array_equal(g, r)
    assert (got[0] == 0).all()


@pytest.mark.parametrize("B,G,V", [(4, 4, 151936), (5, 2, 3001), (1, 0, 100)])
def test_accept_greedy(O, ctx, B, G, V):
    import torch
    rng = np.random.default_rng(V + G)
    tgt = rng.normal(0, 3, (B, G + 1, V)).astype(np.float32)
    am = tgt.argmax(-1)
    drafts = am[:, :G].astype(np.int32).copy()
    if G >= 2:
        drafts[1, 1] = (drafts[1, 1] + 1) % V   # mismatch at position 1
        drafts[0, 0] = (drafts[0, 0] + 7) % V   # mismatch at position 0
    tgt[-1, 0, 5] = tgt[-1, 0].max()             # a tie: first index wins
    acc, out = ctx.accept_greedy(torch.from_numpy(tgt).cuda(),
                                 torch.from_numpy(drafts.reshape(B, G)).cuda())
    racc, rout = O.accept_greedy(tgt, drafts.reshape(B, G))
    assert np.array_equal(acc.cpu().numpy(), racc)
    assert np.array_equal(out.cpu().numpy(), rout)


def test_accept_argument_errors(ctx, pkg):
    import torch
    t = torch.zeros(1, 2, 10, device="cuda")
    d = torch.zeros(1, 1, 10, device="cuda")
    u = torch.zeros(1, 3, device="cuda")
    with pytest.raises(pkg.IfrError, match="temperature"):
        ctx.accept(t, d, u, 0.0)
    with pytest.raises(pkg.IfrError, match="temperature"):
        ctx.accept(t, d, u, float("nan"))


# ---- filtered acceptance (ifr_accept_filtered) vs the oracle's restatement ----

ACCEPT_FILTERS = [  # the sampler tests' filter settings with a positive temperature
    dict(temperature=0.8),
    dict(temperature=0.8, top_k=20),
    dict(temperature=0.8, top_p=0.9),
    dict(temperature=1.0, top_p=0.3),
    dict(temperature=0.8, min_p=0.05),
    dict(temperature=0.6, top_k=50, top_p=0.95, min_p=0.02),
    dict(temperature=1.3, top_k=1),
    dict(temperature=0.8, top_p=0.0),
]


def _run_filtered(ctx, tgt, dft, u, kw):
    import torch
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    kw = dict(kw)
    T = kw.pop("temperature")
    acc, out, dout = ctx.accept_filtered(d(tgt), d(dft), d(u), T, **kw)
    return acc.cpu().numpy(), out.cpu().numpy(), dout.cpu().numpy()


def _oracle_filtered(O, tgt, dft, u, kw):
    kw = dict(kw)
    T = kw.pop("temperature")
    return O.accept_filtered(tgt, dft, u, T, **kw)


@pytest.mark.parametrize("kw", ACCEPT_FILTERS, ids=lambda d: ",".join(f"{k}={v}" for k, v in d.items()))
@pytest.mark.parametrize("B,G,V", [(4, 5, 151936), (6, 3, 5000), (3, 2, 7)])
def test_accept_filtered_bit_exact(O, ctx, kw, B, G, V):
    rng = np.random.default_rng(V + 31 * G + len(kw))
    for noise in (0.5, 2.0):
        tgt, dft, u = _case(rng, B, G, V, noise)
        got = _run_filtered(ctx, tgt, dft, u, kw)
        ref = _oracle_filtered(O, tgt, dft, u, kw)
        for g, r, name in zip(got, ref, ("accept_count", "out_tokens", "draft_tokens")):
            assert np.array_equal(g, r), (name, noise, g, r)


@pytest.mark.parametrize("kw", [ACCEPT_FILTERS[2], ACCEPT_FILTERS[5]],
                         ids=lambda d: ",".join(f"{k}={v}" for k, v in d.items()))
def test_accept_filtered_config3_full_batch(O, ctx, kw):
    """BASELINE config 3's shape (64 x gamma 5 x vocab 151936) with filters"""
    rng = np.random.default_rng(303)
    tgt, dft, u = _case(rng, 64, 5, 151936)
    got = _run_filtered(ctx, tgt, dft, u, kw)
    ref = _oracle_filtered(O, tgt, dft, u, kw)
    for g, r, name in zip(got, ref, ("accept_count", "out_tokens", "draft_tokens")):
        assert np.array_equal(g, r), name


def test_accept_filtered_no_filters_equals_accept(ctx):
    """with every filter off, the filtered entry point gives ifr_accept's
    results (drafts drawn in both)"""
    rng = np.random.default_rng(41)
    tgt, dft, u = _case(rng, 8, 4, 32000)
    u = u * np.float32(0.999) + np.float32(0.0005)
    a = _run(ctx, tgt, dft, u, 0.8)
    b = _run_filtered(ctx, tgt, dft, u, dict(temperature=0.8))
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_accept_filtered_argument_errors(ctx, pkg):
    import torch
    t = torch.zeros(1, 2, 10, device="cuda")
    d = torch.zeros(1, 1, 10, device="cuda")
    u = torch.zeros(1, 3, device="cuda")
    with pytest.raises(pkg.IfrError, match="temperature"):
        ctx.accept_filtered(t, d, u, 0.0)
    with pytest.raises(pkg.IfrError, match="top_p"):
        ctx.accept_filtered(t, d, u, 0.8, top_p=1.5)
    with pytest.raises(pkg.IfrError, match="top_k"):
        ctx.accept_filtered(t, d, u, 0.8, top_k=-1)
    with pytest.raises(pkg.IfrError, match="min_p"):
        ctx.accept_filtered(t, d, u, 0.8, min_p=2.0)
