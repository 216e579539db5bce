"""GPU parity of the dense tensor-core GEMM (ifr_qgemm_dense: tcgen05 MMAs,
fp16 operands, f32 accumulation in tensor memory) through the C ABI.

Two references per case:
  * the stated arithmetic in f64: the oracle's fp16 weights of the dense path
    (oracle.dense_fp16_weights: each weight one rounding from its exact
    integer quant) times fp16(X 2^e) 2^-e (e per column: max|x| 2^e in
    [2^13, 2^14)); only the f32 summation order differs, so the tolerance is
    tight (DENSE_TOL);
  * the exact product of the oracle (f64), within the fp16 rounding of both
    operands (EXACT_TOL).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FORMATS = [12, 13, 14, 8]
NAMES = {12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 8: "Q8_0"}
DENSE_TOL = 2e-5   # norm-relative per column vs the fp16-operand model (f32 sums)
EXACT_TOL = 3e-3   # norm-relative per column vs the exact f64 product


def fp16_model(O, qt, q, M, K, X):
    W16 = O.dense_fp16_weights(qt, q, M, K).astype(np.float64)
    amax = np.abs(X).max(axis=1)
    e = np.zeros(len(X), dtype=np.int64)
    nz = amax > 0
    _, ex = np.frexp(amax[nz])
    e[nz] = 14 - ex
    Xs = (X.astype(np.float64) * np.ldexp(1.0, e)[:, None]).astype(np.float16).astype(np.float64)
    X16 = Xs * np.ldexp(1.0, -e)[:, None]
    return X16 @ W16.T


# (M, K, N): one tile; ragged rows; split-K with partial sums; two column tiles;
# the largest column tile; a column count that is not a multiple of 16
CASES = [(256, 512, 16), (300, 768, 40), (1000, 1024, 9), (512, 2048, 160), (136, 1024, 300),
         (128, 1024, 256), (2048, 4096, 64), (384, 1024, 512), (256, 512, 700)]


@pytest.mark.parametrize("qt", FORMATS)
@pytest.mark.parametrize("M,K,N", CASES)
def test_dense_parity(O, ctx, qt, M, K, N):
    import torch
    rng = np.random.default_rng(M * 13 + K + N + qt)
    q = O.quantize(qt, rng.normal(0, 0.02, (M, K)).astype(np.float32))
    W = ctx.upload(qt, q, M, K)
    X = rng.normal(0, 1, (N, K)).astype(np.float32)
    X[N // 2] *= 1e-3  # columns of very different scale share a tile
    Y = ctx.qgemm_dense(W, torch.from_numpy(X).cuda()).cpu().numpy()
    assert np.isfinite(Y).all(), NAMES[qt]
    err = O.norm_rel(Y, fp16_model(O, qt, q, M, K, X))
    assert err.max() < DENSE_TOL, (NAMES[qt], M, K, N, err.max())
    err = O.norm_rel(Y, O.gemm_ref(qt, q, M, K, X, act=0))
    assert err.max() < EXACT_TOL, (NAMES[qt], M, K, N, err.max())


def test_dense_zero_and_repeat(O, ctx):
    """zero columns give zeros; a second call with other shapes reuses the scratch"""
    import torch
    rng = np.random.default_rng(5)
    M, K = 384, 1024
    q = O.quantize(12, rng.normal(0, 0.02, (M, K)).astype(np.float32))
    W = ctx.upload(12, q, M, K)
    X = rng.normal(0, 1, (33, K)).astype(np.float32)
    X[7] = 0.0
    Y = ctx.qgemm_dense(W, torch.from_numpy(X).cuda()).cpu().numpy()
    assert np.all(Y[7] == 0.0)
    Y2 = ctx.qgemm_dense(W, torch.from_numpy(X[:17].copy()).cuda()).cpu().numpy()
    assert np.allclose(Y2, Y[:17], rtol=0, atol=1e-6 * np.abs(Y).max())
    ctx.sync()


@pytest.mark.parametrize("qt", FORMATS)
@pytest.mark.parametrize("M,K,N", [(300, 768, 40), (512, 2048, 160), (136, 1024, 300), (2048, 4096, 64),
                                   (256, 512, 700)])
def test_dense_fp16_stages_bit_exact(O, ctx, qt, M, K, N):
    """ifr_tensor_prepare_dense: the dense GEMM copying fp16 operand stages
    built once gives bit-for-bit the results of the dequantizing kernel
    (ragged rows, split-K partials, several column tiles)"""
    import torch
    rng = np.random.default_rng(M * 7 + K + N + qt)
    q = O.quantize(qt, rng.normal(0, 0.02, (M, K)).astype(np.float32))
    W = ctx.upload(qt, q, M, K)
    X = torch.from_numpy(rng.normal(0, 1, (N, K)).astype(np.float32)).cuda()
    Y0 = ctx.qgemm_dense(W, X).cpu().numpy()
    ctx.prepare_dense(W)
    Y1 = ctx.qgemm_dense(W, X).cpu().numpy()
    assert np.array_equal(Y0.view(np.uint32), Y1.view(np.uint32)), (NAMES[qt], M, K, N)
