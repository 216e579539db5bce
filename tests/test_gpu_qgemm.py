"""GPU parity: bit-exact dequantization and the small-N verify GEMV against
the CPU oracle, through the C ABI (libinferno_b200.so)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FORMATS = [12, 13, 14, 8]
NAMES = {12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 8: "Q8_0"}
# norm-relative error per output column against the oracle with the same
# activation semantics (Q8_K for the K-quants, f32 for Q8_0): the GPU sums
# exact integer (or exact fp16-split) products and accumulates in f32
TOL = 2e-6


def _torch():
    import torch
    return torch


def random_valid_blocks(O, rng, qt, rows, cols):
    be, bb = O.BLOCK[qt]
    nb = rows * cols // be
    blk = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    f16 = lambda: np.asarray(rng.normal(0, 0.01, nb), np.float16).view(np.uint8).reshape(nb, 2)  # noqa: E731
    if qt in (12, 13):
        blk[:, 0:2] = f16()
        blk[:, 2:4] = f16()
    elif qt == 14:
        blk[:, 208:210] = f16()
    else:
        blk[:, 0:2] = f16()
    return blk.ravel()


@pytest.mark.parametrize("qt", FORMATS)
def test_dequant_bit_exact(O, ctx, qt):
    rng = np.random.default_rng(qt)
    for rows, cols in ((16, 1024), (37, 2048)):
        q = random_valid_blocks(O, rng, qt, rows, cols)
        W = ctx.upload(qt, q, rows, cols)
        got = ctx.dequant(W).cpu().numpy().ravel()
        ref = O.dequantize(qt, q, rows * cols)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), NAMES[qt]
    # encoder-made weights, and the golden gguf-py blocks
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "dequant_golden.npz"))
    be, _ = O.BLOCK[qt]
    cols = 256 if qt != 8 else 32
    W = ctx.upload(qt, g[f"{NAMES[qt]}_blocks"], 64 * be // cols, cols)
    got = ctx.dequant(W).cpu().numpy().ravel()
    assert np.array_equal(got.view(np.uint32), g[f"{NAMES[qt]}_gguf_py"].view(np.uint32))


# (96, 3584), (130, 4096), (64, 12288): few row groups over several K passes
SHAPES = [(256, 256), (1000, 1024), (96, 3584), (130, 4096), (64, 12288)]


@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("qt", FORMATS)
@pytest.mark.parametrize("M,K", SHAPES)
def test_qgemm_parity(O, ctx, qt, M, K, act):
    torch = _torch()
    rng = np.random.default_rng(M * 7 + K + qt)
    q = O.quantize(qt, rng.normal(0, 0.02, (M, K)).astype(np.float32))
    W = ctx.upload(qt, q, M, K)
    X = rng.normal(0, 1, (8, K)).astype(np.float32)
    ref = O.gemm_ref(qt, q, M, K, X, act=act)
    Xd = torch.from_numpy(X).cuda()
    ctx.set_activation(act)
    try:
        for n in (1, 2, 3, 4, 5, 8):
            Y = ctx.qgemm(W, Xd[:n].contiguous()).cpu().numpy()
            err = O.norm_rel(Y, ref[:n])
            assert err.max() < TOL, (NAMES[qt], M, K, n, act, err)
    finally:
        ctx.set_activation(0)


def _rmsnorm(X, w, eps):
    """rmsnorm_cpu! (src/ModelCPU.jl:111-123) per column, in f32"""
    ss = np.einsum("ij,ij->i", X.astype(np.float64), X.astype(np.float64)).astype(np.float32)
    scale = (np.float32(1.0) / np.sqrt(ss / np.float32(X.shape[1]) + np.float32(eps))).astype(np.float32)
    return (X * scale[:, None] * w[None, :]).astype(np.float32)


# (12, 32, 20480): the folded norm's sums of squares over ten K passes
NORM_CASES = [(12, 256, 256), (12, 1000, 1024), (13, 130, 4096), (14, 300, 2048), (8, 256, 1024),
              (8, 200, 1152), (8, 64, 800), (12, 32, 20480)]


@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("qt,M,K", NORM_CASES)
def test_qgemm_rmsnorm_parity(O, ctx, qt, M, K, act):
    """ifr_qgemm_rmsnorm = RMSNorm then GEMV: exact activations fold the norm
    into the epilogue (the oracle normalises first, so only f32 rounding
    differs: TOL); Q8_K activations quantize the normalised input like the
    reference (a rare rounding flip of one Q8_K value moves a column by
    ~1e-4: Q8K_TOL).  Ragged K (Q8_0, K = 800, 1152) takes the scalar loads."""
    torch = _torch()
    rng = np.random.default_rng(M + K * 3 + qt + act)
    q = O.quantize(qt, rng.normal(0, 0.02, (M, K)).astype(np.float32))
    W = ctx.upload(qt, q, M, K)
    X = rng.normal(0, 1, (13, K)).astype(np.float32)
    X[3] *= 40.0  # columns of very different scale
    w = (1.0 + rng.normal(0, 0.2, K)).astype(np.float32)
    eps = 1e-6
    ref = O.gemm_ref(qt, q, M, K, _rmsnorm(X, w, eps), act=act if qt != 8 else 0)
    Xd = torch.from_numpy(X).cuda()
    wd = torch.from_numpy(w).cuda()
    tol = TOL if act == 0 or qt == 8 else 1e-3
    ctx.set_activation(act)
    try:
        for n in (1, 5, 8, 13):
            Y = ctx.qgemm_rmsnorm(W, Xd[:n].contiguous(), wd, eps).cpu().numpy()
            err = O.norm_rel(Y, ref[:n])
            assert err.max() < 5 * tol, (NAMES[qt], M, K, n, act, err)
    finally:
        ctx.set_activation(0)


@pytest.mark.parametrize("qt", FORMATS)
def test_qgemm_matches_reference_c_kernel(O, ctx, qt):
    """in the reference's activation mode (Q8_K) the GPU GEMV reproduces the
    outputs of the reference's own quant_kernels.c (golden vectors made by
    tests/golden/gen_golden.py) up to the C kernel's f32 summation order"""
    import os
    torch = _torch()
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "gemv_golden.npz"))
    M, K = int(g["M"]), int(g["K"])
    W = ctx.upload(qt, g[f"{NAMES[qt]}_W"], M, K)
    ctx.set_activation(1)
    try:
        Y = ctx.qgemm(W, torch.from_numpy(np.ascontiguousarray(g["X"])).cuda()).cpu().numpy()
    finally:
        ctx.set_activation(0)
    assert O.norm_rel(Y, g[f"{NAMES[qt]}_ref"]).max() < 1e-5


@pytest.mark.parametrize("qt", FORMATS)
def test_qgemm_random_blocks_and_scales(O, ctx, qt):
    """raw random blocks (all scale/min bit patterns) and activations spanning
    many binades, a zero column and a column of one huge element"""
    torch = _torch()
    rng = np.random.default_rng(100 + qt)
    M, K = 200, 2048
    q = random_valid_blocks(O, rng, qt, M, K)
    W = ctx.upload(qt, q, M, K)
    X = rng.normal(0, 1, (6, K)).astype(np.float32)
    X[1] *= 1e-20
    X[2] *= 1e20
    X[3] = 0.0
    X[4] = 0.0
    X[4, 777] = 3e4
    X[5] *= np.exp(rng.normal(0, 4, K)).astype(np.float32)
    ref = O.gemm_ref(qt, q, M, K, X)
    Y = ctx.qgemm(W, torch.from_numpy(X).cuda()).cpu().numpy()
    assert np.all(Y[3] == 0.0)
    keep = [0, 1, 2, 4, 5]
    err = O.norm_rel(Y[keep], ref[keep])
    assert err.max() < 1e-5, (NAMES[qt], err)


def test_qgemm_q8_0_ragged_k(O, ctx):
    """Q8_0 with K not a multiple of 256 (the config-5 draft has 1152)"""
    torch = _torch()
    rng = np.random.default_rng(5)
    for M, K in ((77, 1152), (64, 32), (33, 288)):
        q = O.quantize(8, rng.normal(0, 0.02, (M, K)).astype(np.float32))
        W = ctx.upload(8, q, M, K)
        X = rng.normal(0, 1, (5, K)).astype(np.float32)
        Y = ctx.qgemm(W, torch.from_numpy(X).cuda()).cpu().numpy()
        assert O.norm_rel(Y, O.gemm_ref(8, q, M, K, X)).max() < TOL


def test_qgemm_many_columns(O, ctx):
    """more than 8 columns run in passes of 8"""
    torch = _torch()
    rng = np.random.default_rng(6)
    M, K = 300, 1024
    q = O.quantize(12, rng.normal(0, 0.02, (M, K)).astype(np.float32))
    W = ctx.upload(12, q, M, K)
    X = rng.normal(0, 1, (19, K)).astype(np.float32)
    Y = ctx.qgemm(W, torch.from_numpy(X).cuda()).cpu().numpy()
    assert O.norm_rel(Y, O.gemm_ref(12, q, M, K, X)).max() < TOL


@pytest.mark.parametrize("qt", FORMATS)
def test_qgemm_full_size_sampled_rows(O, ctx, qt):
    """BASELINE sweep shape 151936 x 4096 at N=5: rows sampled across the
    whole matrix (first, last, random) checked against the oracle"""
    torch = _torch()
    rng = np.random.default_rng(200 + qt)
    M, K = 151936, 4096
    rb = O.row_bytes(qt, K)
    # encode a 4096-row pool and tile it (keeps the CPU encoder fast)
    pool = O.quantize(qt, rng.normal(0, 0.02, (4096, K)).astype(np.float32)).reshape(4096, rb)
    idx = rng.integers(0, 4096, M)
    q = pool[idx].ravel()
    W = ctx.upload(qt, q, M, K)
    X = rng.normal(0, 1, (5, K)).astype(np.float32)
    Y = ctx.qgemm(W, torch.from_numpy(X).cuda()).cpu().numpy()
    rows = np.unique(np.concatenate([[0, 1, 15, 16, M - 1, M - 16], rng.integers(0, M, 200)]))
    ref = O.gemm_ref(qt, pool[idx[rows]].ravel(), len(rows), K, X)
    err = O.norm_rel(Y[:, rows], ref)
    assert err.max() < TOL, (NAMES[qt], err)
    del W


def test_legacy_shims(O, pkg):
    """the reference's own symbols (host pointers) through quantized_kernels"""
    import importlib
    qk = importlib.import_module("inferno_b200.quantized_kernels")
    rng = np.random.default_rng(8)
    M, K = 123, 1024
    for qt, fn in ((12, qk.q4_k_gemv_), (13, qk.q5_k_gemv_), (14, qk.q6_k_gemv_), (8, qk.q8_0_gemv_)):
        q = O.quantize(qt, rng.normal(0, 0.02, (M, K)).astype(np.float32))
        x = rng.normal(0, 1, K).astype(np.float32)
        out = np.zeros(M, np.float32)
        fn(out, q, x, K, M)
        # the shims keep the reference's own activation rounding (Q8_K)
        assert O.norm_rel(out, O.gemm_ref(qt, q, M, K, x, act=1)[0]).max() < TOL


def test_argument_errors(O, ctx, pkg):
    import ctypes
    L = pkg.load()
    rng = np.random.default_rng(9)
    q = O.quantize(12, rng.normal(0, 0.02, (4, 256)).astype(np.float32))
    h = ctypes.c_void_p()
    qp = q.ctypes.data_as(ctypes.c_void_p)
    assert L.ifr_weights_upload(ctx.handle, 12, qp, 4, 250, ctypes.byref(h)) == 1   # cols % 256
    assert b"multiple" in L.ifr_last_error()
    assert L.ifr_weights_upload(ctx.handle, 3, qp, 4, 256, ctypes.byref(h)) == 1    # type
    assert b"unsupported weight type" in L.ifr_last_error()
    assert L.ifr_weights_upload(ctx.handle, 12, qp, 0, 256, ctypes.byref(h)) == 1   # rows
    W = ctx.upload(12, q, 4, 256)
    assert L.ifr_qgemm(ctx.handle, W.handle, ctypes.c_void_p(16), 0, ctypes.c_void_p(16)) == 1


# tall matrices (>= 2 x 148 groups of 15 row blocks): the row-block-per-warp
# kernel, which keeps every unit's fragments in shared memory (K = 1024, and
# K = 4096 with Q8_K activations); exact Q4_K / Q5_K activations as int8
# limbs; exact activations whose fragments leave too little room split K over
# CTA pairs (half the fragments each, the second half's partials added by a
# second kernel); Q8_0 at K = 4096 (larger tiles) and Q4_K with Q8_K
# activations take the unit-split kernel
TALL = [(12, 1024), (13, 1024), (14, 1024), (8, 1024), (12, 4096), (13, 4096), (14, 4096), (8, 4096)]


@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("qt,K", TALL)
def test_qgemm_tall(O, ctx, qt, K, act):
    torch = _torch()
    M = 71040 + 37  # ragged last row block and group
    rng = np.random.default_rng(qt * 31 + K)
    pool = O.quantize(qt, rng.normal(0, 0.02, (512, K)).astype(np.float32))
    rb = pool.size // 512
    q = pool.reshape(512, rb)[np.arange(M) % 512].ravel()
    W = ctx.upload(qt, q, M, K)
    X = rng.normal(0, 1, (8, K)).astype(np.float32)
    a = act if qt != 8 else 0  # Q8_0 is always exact
    ref = O.gemm_ref(qt, pool, 512, K, X, act=a)  # rows repeat with period 512
    idx = np.arange(M) % 512
    Xd = torch.from_numpy(X).cuda()
    ctx.set_activation(act)
    try:
        for n in (1, 2, 3, 5, 6, 8):
            Y = ctx.qgemm(W, Xd[:n].contiguous()).cpu().numpy()
            err = O.norm_rel(Y, ref[:n][:, idx])
            assert err.max() < TOL, (NAMES[qt], K, n, act, err)
        w = (1.0 + rng.normal(0, 0.2, K)).astype(np.float32)
        Yn = ctx.qgemm_rmsnorm(W, Xd[:5].contiguous(), torch.from_numpy(w).cuda(), 1e-6).cpu().numpy()
        refn = O.gemm_ref(qt, pool, 512, K, _rmsnorm(X[:5], w, 1e-6), act=a)
        assert O.norm_rel(Yn, refn[:, idx]).max() < 5 * (TOL if a == 0 else 1e-3)
    finally:
        ctx.set_activation(0)


@pytest.mark.parametrize("qt", [12, 13, 14])
def test_qgemm_tall_exact_outlier_channels(O, ctx, qt):
    """exact activations with a few massive channels (200x the others): the
    Q4_K / Q5_K tall kernel writes each unit of a column as three int8 limbs
    over the unit's amax, so small elements beside an outlier keep ~6e-8 of
    that amax (Q6_K keeps the fp16 hi/lo split); still within TOL of the
    oracle's f32 dot products"""
    torch = _torch()
    M, K = 71040 + 5, 4096
    rng = np.random.default_rng(qt + 777)
    pool = O.quantize(qt, rng.normal(0, 0.02, (512, K)).astype(np.float32))
    rb = pool.size // 512
    idx = np.arange(M) % 512
    W = ctx.upload(qt, pool.reshape(512, rb)[idx].ravel(), M, K)
    X = rng.normal(0, 1, (8, K)).astype(np.float32)
    X[:, [5, 1300, 4000]] *= 200.0
    X[3, 700:956] = 0.0          # an all-zero unit of one column
    X[6, 2048:2304] *= 1e-30     # a unit of tiny values (its own scale)
    ref = O.gemm_ref(qt, pool, 512, K, X, act=0)
    ctx.set_activation(0)
    Xd = torch.from_numpy(X).cuda()
    for n in (1, 5, 8):
        Y = ctx.qgemm(W, Xd[:n].contiguous()).cpu().numpy()
        err = O.norm_rel(Y, ref[:n][:, idx])
        assert err.max() < TOL, (NAMES[qt], n, err)
