"""Filtered sampling (CommonOps.softmax_sample_scratch!, src/CommonOps.jl:196-318)
and the presence / repetition penalties (src/ModelCPU.jl:1202-1238,
src/CommonOps.jl:63-76).

CPU: the oracle against the reference's own known answers
(tests/unit/test_common_ops.jl:66-146, tests/unit/test_speculative_decoding.jl).
Those tests draw with Julia's rand(); here the uniforms are supplied, so each
property is checked over a grid of uniforms instead.
GPU: ifr_sample / ifr_apply_penalties through the C ABI, bit-exact with the
oracle for the same logits and uniforms."""
import numpy as np
import pytest

GRID = np.linspace(0.0, 0.999, 400).astype(np.float32)


def _set(O, logits, **kw):
    l = np.asarray(logits, np.float32)
    return set(O.sample(np.tile(l, (len(GRID), 1)), GRID, **kw).tolist())


# ---- the reference's known answers, on the oracle ------------------------------

def test_filter_boundaries(O):
    # top_p = 0 keeps the argmax alone (test_common_ops.jl:121)
    assert _set(O, [0, 1, 2], top_p=0.0) == {2}
    # top_k = 2 of [0,1,2,3]: only the two largest (:123-127)
    assert _set(O, [0, 1, 2, 3], top_k=2) == {2, 3}
    # top_k = n disables the filter (:129-132)
    assert _set(O, [0, 0, 0, 0], top_k=4) == {0, 1, 2, 3}
    # top_p = 0.5 over (0.2, 0.31, 0.49): 0.49 < 0.5, so 0.31 joins (:134-139)
    assert _set(O, np.log(np.array([0.2, 0.31, 0.49], np.float32)), top_p=0.5) == {1, 2}
    # min_p = 1 with equal logits keeps all of them (:141-145)
    assert _set(O, [0, 0, 0, 0], min_p=1.0) == {0, 1, 2, 3}


def test_tiny_temperature_and_non_finite(O):
    # temperature 1e-30 with top_k = 1 is the argmax (:66-74)
    assert _set(O, [0, 1, 2], temperature=1e-30, top_k=1) == {2}
    # -Inf logits are impossible; top_k = 2 of [-Inf, 0, -Inf, 1] (:77-83)
    assert _set(O, [-np.inf, 0, -np.inf, 1], top_k=2) == {1, 3}
    # every logit -Inf: the first token (:85-86)
    assert O.sample(np.array([[-np.inf, -np.inf]], np.float32), [0.5]).tolist() == [0]
    assert O.sample(np.array([[-np.inf, -np.inf]], np.float32), [0.5], top_p=0.5, top_k=1).tolist() == [0]
    # +Inf and NaN are rejected (:88-95): token -1 here
    assert O.sample(np.array([[1, np.inf]], np.float32), [0.5]).tolist() == [-1]
    assert O.sample(np.array([[1, np.nan]], np.float32), [0.5]).tolist() == [-1]
    # temperature 0: argmax, first index on ties
    assert O.sample(np.array([[0, 3, 3, 1]], np.float32), [0.9], temperature=0.0).tolist() == [1]


def test_sampler_frequencies(O):
    """without filters the draws follow softmax(l / T)"""
    rng = np.random.default_rng(0)
    l = rng.normal(0, 1, 50).astype(np.float32)
    u = rng.random(20000, dtype=np.float32)
    t = O.sample(np.tile(l, (len(u), 1)), u, temperature=0.8)
    p = np.exp(l / 0.8)
    p /= p.sum()
    f = np.bincount(t, minlength=50) / len(u)
    assert np.abs(f - p).max() < 0.02


def test_filters_compose(O):
    """top-k, then top-p on the renormalised top-k mass, then min-p (:217-299)"""
    rng = np.random.default_rng(5)
    l = rng.normal(0, 2, 300).astype(np.float32)
    T, k, p, mp = 0.7, 40, 0.8, 0.05
    order = np.argsort(-l, kind="stable")
    e = np.exp((l - l.max()) / T)
    keep = np.zeros(300, bool)
    keep[order[:k]] = True
    pk = np.where(keep, e, 0)
    pk = pk / pk.sum()
    o2 = np.argsort(-pk, kind="stable")
    cut = np.searchsorted(np.cumsum(pk[o2]), p) + 1
    keep2 = np.zeros(300, bool)
    keep2[o2[:cut]] = True
    keep2 &= pk >= pk.max() * mp
    got = _set(O, l, temperature=T, top_k=k, top_p=p, min_p=mp)
    assert got <= set(np.nonzero(keep2)[0].tolist())
    assert len(got) >= keep2.sum() - 2  # the grid reaches (nearly) every kept token


def test_penalties_oracle(O):
    x = np.array([[1.0, -2.0, 0.0, 3.0]], np.float32)
    y = O.apply_penalties(x, [[0, 1, 2, 0, -1, 7]], presence=0.5, repetition=2.0)
    # presence first (l - 0.5), then repetition (/2 if > 0 else *2); duplicates,
    # -1 and out-of-range ids are ignored
    assert y.tolist() == [[0.25, -5.0, -1.0, 3.0]]
    assert np.array_equal(O.apply_penalties(x, [[0, 1]], 0.0, 1.0), x)


def test_sample_abi_argument_errors(pkg):
    """argument checks happen on the host, before any device work"""
    import ctypes
    L = pkg.load()
    c = ctypes.c_void_p(1)  # never dereferenced: every call below fails its checks first
    buf = ctypes.c_void_p(8)
    bad = [
        dict(temperature=-1.0), dict(temperature=float("nan")), dict(temperature=float("inf")),
        dict(top_p=-0.1), dict(top_p=1.1), dict(top_p=float("nan")), dict(top_k=-1),
        dict(min_p=-0.1), dict(min_p=1.1), dict(min_p=float("nan")), dict(vocab=0),
    ]
    for b in bad:
        a = dict(temperature=1.0, top_k=0, top_p=1.0, min_p=0.0, vocab=4)
        a.update(b)
        rc = L.ifr_sample(c, buf, 1, a["vocab"], ctypes.c_float(a["temperature"]), a["top_k"],
                          ctypes.c_float(a["top_p"]), ctypes.c_float(a["min_p"]), buf, buf)
        assert rc == 1, b  # IFR_ERR_ARG
    assert L.ifr_apply_penalties(c, buf, 1, 4, buf, 1, ctypes.c_float(0.0), ctypes.c_float(0.0)) == 1


# ---- GPU parity -----------------------------------------------------------------

def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _gpu_sample(ctx, logits, u, **kw):
    return ctx.sample(_dev(logits), _dev(u), **kw).cpu().numpy()


FILTERS = [
    dict(temperature=0.8),
    dict(temperature=0.8, top_k=20),
    dict(temperature=0.8, top_p=0.9),
    dict(temperature=1.0, top_p=0.3),
    dict(temperature=0.8, min_p=0.05),
    dict(temperature=0.6, top_k=50, top_p=0.95, min_p=0.02),
    dict(temperature=1.3, top_k=1),
    dict(temperature=0.0),
    dict(temperature=0.8, top_p=0.0),
]


@pytest.mark.gpu
@pytest.mark.parametrize("V", [7, 2048, 5000, 151936, 262144])
@pytest.mark.parametrize("kw", FILTERS, ids=lambda d: ",".join(f"{k}={v}" for k, v in d.items()))
def test_sample_bit_exact(O, ctx, V, kw):
    rng = np.random.default_rng(V + 7 * len(kw))
    rows = 6 if V > 200000 else (12 if V > 100000 else 24)
    logits = rng.normal(0, 3, (rows, V)).astype(np.float32)
    u = rng.random(rows, dtype=np.float32)
    u[0] = 0.0
    u[1] = np.float32(0.99999994)
    got = _gpu_sample(ctx, logits, u, **kw)
    ref = O.sample(logits, u, **kw)
    assert np.array_equal(got, ref), (got, ref)


@pytest.mark.gpu
def test_sample_ties_and_edges(O, ctx):
    """equal values at the top-k and top-p cuts (lower ids win), -Inf, NaN/+Inf
    rows, a single-token vocabulary, all -Inf"""
    V = 4099
    rows = []
    r = np.zeros(V, np.float32)
    rows.append(r.copy())                       # all equal: ties everywhere
    r = np.full(V, -np.inf, np.float32)
    r[[5, 900, 4000]] = [1.0, 1.0, 0.5]         # mostly -Inf
    rows.append(r)
    r = np.round(np.random.default_rng(1).normal(0, 1, V) * 2) / 2
    rows.append(r.astype(np.float32))           # many repeated values
    r = np.zeros(V, np.float32)
    r[17] = np.nan
    rows.append(r)                              # NaN -> -1
    r = np.zeros(V, np.float32)
    r[3000] = np.inf
    rows.append(r)                              # +Inf -> -1
    rows.append(np.full(V, -np.inf, np.float32))  # all -Inf -> 0
    L = np.stack(rows)
    u = np.linspace(0.0, 0.99, len(rows)).astype(np.float32)
    for kw in [dict(top_k=7), dict(top_k=3000), dict(top_p=0.5), dict(top_p=0.001), dict(min_p=0.9),
               dict(top_k=100, top_p=0.7, min_p=0.1), dict()]:
        for uu in (u, u[::-1].copy()):
            got = _gpu_sample(ctx, L, uu, **kw)
            ref = O.sample(L, uu, **kw)
            assert np.array_equal(got, ref), (kw, got, ref)
    one = np.array([[2.5], [-1.0]], np.float32)
    assert _gpu_sample(ctx, one, np.array([0.3, 0.7], np.float32)).tolist() == [0, 0]


@pytest.mark.gpu
def test_sample_known_answers_gpu(O, ctx):
    """the reference's filter-boundary answers (test_common_ops.jl:119-146) on the device"""
    def gset(l, **kw):
        l = np.asarray(l, np.float32)
        return set(_gpu_sample(ctx, np.tile(l, (len(GRID), 1)), GRID, **kw).tolist())
    assert gset([0, 1, 2], top_p=0.0) == {2}
    assert gset([0, 1, 2, 3], top_k=2) == {2, 3}
    assert gset([0, 0, 0, 0], top_k=4) == {0, 1, 2, 3}
    assert gset(np.log(np.array([0.2, 0.31, 0.49], np.float32)), top_p=0.5) == {1, 2}
    assert gset([0, 0, 0, 0], min_p=1.0) == {0, 1, 2, 3}
    assert gset([-np.inf, 0, -np.inf, 1], top_k=2) == {1, 3}


@pytest.mark.gpu
def test_penalties_bit_exact(O, ctx):
    import torch
    rng = np.random.default_rng(9)
    rows, V, n = 5, 151936, 300
    logits = rng.normal(0, 3, (rows, V)).astype(np.float32)
    seen = rng.integers(-2, V + 3, (rows, n)).astype(np.int32)
    seen[:, 10:20] = seen[:, :10]  # duplicates are penalised once
    for pres, rep in [(0.5, 1.3), (0.0, 1.2), (0.7, 1.0), (-0.25, 0.8)]:
        d = torch.from_numpy(logits.copy()).cuda()
        ctx.apply_penalties(d, _dev(seen), pres, rep)
        got = d.cpu().numpy()
        ref = O.apply_penalties(logits, seen, pres, rep)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (pres, rep)
    # penalties then sampling, as the reference's generate loop does (ModelCPU.jl:1236-1242)
    d = torch.from_numpy(logits.copy()).cuda()
    ctx.apply_penalties(d, _dev(seen), 0.5, 1.3)
    u = rng.random(rows, dtype=np.float32)
    got = ctx.sample(d, _dev(u), temperature=0.8, top_k=40, top_p=0.95).cpu().numpy()
    ref = O.sample(O.apply_penalties(logits, seen, 0.5, 1.3), u, temperature=0.8, top_k=40, top_p=0.95)
    assert np.array_equal(got, ref)


# ---- filtered speculative acceptance (oracle restatement) -----------------------

def test_accept_filtered_without_filters_is_accept(O):
    """with every filter off the filtered verification is the plain one"""
    rng = np.random.default_rng(3)
    B, G, V = 4, 3, 5000
    tgt = rng.normal(0, 3, (B, G + 1, V)).astype(np.float32)
    dft = (tgt[:, :G] + rng.normal(0, 1, (B, G, V))).astype(np.float32)
    u = rng.random((B, 2 * G + 1), dtype=np.float32) * 0.999 + 0.0005
    got = O.accept_filtered(tgt, dft, u, 0.8)
    ref = O.accept(tgt, dft, u, 0.8)
    for g, r in zip(got, ref):
        assert np.array_equal(g, r)


def _filtered_probs(l, T, top_k, top_p, min_p):
    """the filtered, renormalised distribution in float64 (no ties assumed)"""
    l = np.asarray(l, np.float64)
    keep = np.ones(len(l), bool)
    if 0 < top_k < len(l):
        keep[:] = False
        keep[np.argsort(-l, kind="stable")[:top_k]] = True
    e = np.where(keep, np.exp((l - l.max()) / T), 0.0)
    p = e / e.sum()
    if top_p < 1:
        o = np.argsort(-p, kind="stable")
        m = int(np.searchsorted(np.cumsum(p[o]), top_p)) + 1
        k2 = np.zeros(len(l), bool)
        k2[o[:m]] = True
        p = np.where(k2, p, 0.0)
        p /= p.sum()
    if min_p > 0:
        p = np.where(p >= p.max() * min_p, p, 0.0)
        p /= p.sum()
    return p


def test_accept_filtered_emits_the_filtered_target(O):
    """speculative sampling on filtered distributions leaves the first emitted
    token distributed as the filtered target (drafts from the filtered draft)"""
    rng = np.random.default_rng(11)
    V, T, kw = 16, 0.9, dict(top_k=9, top_p=0.9, min_p=0.03)
    t = rng.normal(0, 1.5, V).astype(np.float32)
    d = (t + rng.normal(0, 1.0, V)).astype(np.float32)
    n = 40000
    tgt = np.broadcast_to(t, (n, 2, V)).copy()
    dft = np.broadcast_to(d, (n, 1, V)).copy()
    u = rng.random((n, 3), dtype=np.float32) * 0.9998 + 0.0001
    acc, out, drafts = O.accept_filtered(tgt, dft, u, T, **kw)
    pt = _filtered_probs(t, T, **kw)
    pd = _filtered_probs(d, T, **kw)
    f0 = np.bincount(out[:, 0], minlength=V) / n
    fd = np.bincount(drafts[:, 0], minlength=V) / n
    assert np.abs(fd - pd).max() < 0.015, (fd, pd)
    assert np.abs(f0 - pt).max() < 0.015, (f0, pt)
    assert np.all(f0[pt == 0] == 0)  # nothing the target's filters drop is emitted
