"""Generate the committed golden fixtures for the verify path.

Run in a container that has gguf-py (0.19.0) and the reference's native kernels
built by `make -C oracle` (oracle/_ref/libquant_ref.so); the outputs are small
.npz/.json files committed beside this script, so the tests never need either.

  dequant_golden.npz  random valid blocks of Q4_K/Q5_K/Q6_K/Q8_0 and their
                      dequantization by gguf-py (gguf.quants.dequantize), an
                      implementation independent of both the reference's
                      src/Dequant.jl and this repo's oracle; plus hand-built
                      known-answer blocks with values computed by hand below.
  gemv_golden.npz     a seeded Q4_K/Q5_K/Q6_K/Q8_0 weight, 3 activation columns
                      and the outputs of the reference's own C kernels
                      (src/kernels/quant_kernels.c q*_gemv, one column per call)
  sampler_golden.json the known answers of tests/unit/test_speculative_decoding.jl:13-46
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402


def f16bytes(v):
    return np.atleast_1d(np.asarray(v, dtype=np.float16)).view(np.uint8)


def random_blocks(rng, qt, nb):
    be, bb = O.BLOCK[qt]
    blk = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    dvals = lambda: f16bytes(rng.normal(0, 0.01, nb)).reshape(nb, 2)  # noqa: E731
    if qt in (O.Q4_K, O.Q5_K):
        blk[:, 0:2] = dvals()
        blk[:, 2:4] = dvals()
    elif qt == O.Q6_K:
        blk[:, 208:210] = dvals()
    else:
        blk[:, 0:2] = dvals()
    return blk.ravel()


def known_answer_blocks():
    """One block per format with d = 1.0 (f16 0x3c00) and chosen fields; the
    expected values are written out from the block layout by hand."""
    cases = {}
    # Q4_K: d=1, dmin=0.5, sc[j]=j+1, m[j]=j (all < 16 so no high bits), nibble = l % 16
    b = np.zeros(144, np.uint8)
    b[0:2] = f16bytes(1.0)
    b[2:4] = f16bytes(0.5)
    sc = [j + 1 for j in range(8)]
    mn = [j for j in range(8)]
    for j in range(4):
        b[4 + j] = sc[j]
        b[8 + j] = mn[j]
    for j in range(4, 8):
        b[8 + j] = (sc[j] & 15) | ((mn[j] & 15) << 4)
    for j in range(4):
        for l in range(32):
            b[16 + 32 * j + l] = (l % 16) | (((l + 3) % 16) << 4)
    exp = np.zeros(256, np.float32)
    for j in range(4):
        for l in range(32):
            exp[64 * j + l] = 1.0 * sc[2 * j] * (l % 16) - 0.5 * mn[2 * j]
            exp[64 * j + 32 + l] = 1.0 * sc[2 * j + 1] * ((l + 3) % 16) - 0.5 * mn[2 * j + 1]
    cases["Q4_K"] = (b, exp)
    # Q5_K: same scales, high bit set for odd l on the low nibble half
    b5 = np.zeros(176, np.uint8)
    b5[0:16] = b[0:16]
    for l in range(32):
        bits = 0
        for j in range(4):
            if l % 2 == 1:
                bits |= 1 << (2 * j)
        b5[16 + l] = bits
    b5[48:176] = b[16:144]
    exp5 = exp.copy()
    for j in range(4):
        for l in range(32):
            if l % 2 == 1:
                exp5[64 * j + l] = 1.0 * sc[2 * j] * ((l % 16) + 16) - 0.5 * mn[2 * j]
    cases["Q5_K"] = (b5, exp5)
    # Q6_K: d=1, scale[g] = g - 8, q6 = (e % 64) -> value (q6 - 32) * scale
    b6 = np.zeros(210, np.uint8)
    q6 = np.array([(e * 7) % 64 for e in range(256)])
    for n in range(2):
        for l in range(32):
            q1, q2, q3, q4 = (q6[128 * n + l], q6[128 * n + 32 + l],
                              q6[128 * n + 64 + l], q6[128 * n + 96 + l])
            b6[64 * n + l] = (q1 & 15) | ((q3 & 15) << 4)
            b6[64 * n + 32 + l] = (q2 & 15) | ((q4 & 15) << 4)
            b6[128 + 32 * n + l] = (q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)
    scl = np.array([g - 8 for g in range(16)], np.int8)
    b6[192:208] = scl.view(np.uint8)
    b6[208:210] = f16bytes(1.0)
    exp6 = np.array([(q6[e] - 32) * scl[e // 16] for e in range(256)], np.float32)
    cases["Q6_K"] = (b6, exp6)
    # Q8_0: d=1, q = i - 16
    b8 = np.zeros(34, np.uint8)
    b8[0:2] = f16bytes(1.0)
    b8[2:34] = np.array([i - 16 for i in range(32)], np.int8).view(np.uint8)
    cases["Q8_0"] = (b8, np.array([i - 16 for i in range(32)], np.float32))
    return cases


def main():
    import gguf
    from gguf import GGMLQuantizationType as QT
    qmap = {O.Q4_K: QT.Q4_K, O.Q5_K: QT.Q5_K, O.Q6_K: QT.Q6_K, O.Q8_0: QT.Q8_0}
    rng = np.random.default_rng(20261201)
    arrays = {}
    for qt in (O.Q4_K, O.Q5_K, O.Q6_K, O.Q8_0):
        name = O.TYPE_NAMES[qt]
        blocks = random_blocks(rng, qt, 64)
        deq = gguf.quants.dequantize(blocks, qmap[qt]).astype(np.float32).ravel()
        arrays[f"{name}_blocks"] = blocks
        arrays[f"{name}_gguf_py"] = deq
    for name, (blk, exp) in known_answer_blocks().items():
        arrays[f"{name}_ka_block"] = blk
        arrays[f"{name}_ka_expected"] = exp
    np.savez_compressed(os.path.join(HERE, "dequant_golden.npz"), **arrays)

    # reference C kernels on a small seeded GEMV
    M, K = 96, 512
    W = rng.normal(0, 0.02, (M, K)).astype(np.float32)
    X = rng.normal(0, 1, (3, K)).astype(np.float32)
    g = {"X": X, "M": np.int64(M), "K": np.int64(K)}
    for qt in (O.Q4_K, O.Q5_K, O.Q6_K, O.Q8_0):
        name = O.TYPE_NAMES[qt]
        q = O.quantize(qt, W)
        g[f"{name}_W"] = q
        g[f"{name}_ref"] = np.stack([O.ref_gemv(qt, q, M, K, X[n]) for n in range(3)])
    np.savez_compressed(os.path.join(HERE, "gemv_golden.npz"), **g)

    sampler = {
        "source": "tests/unit/test_speculative_decoding.jl:13-46 (reference)",
        "sample_from_probs": [
            {"probs": [0.0, 0.0, 1.0, 0.0], "expect": 3},
            {"probs": [1.0, 0.0, 0.0, 0.0], "expect": 1},
            {"probs": [1.0], "expect": 1},
            {"probs": [0.0, 0.0, 0.0], "expect": 3},
        ],
        "argmax_greedy": {"source": "tests/unit/test_common_ops.jl:121 (temperature=0 -> argmax)",
                          "logits": [0.0, 1.0, 2.0], "expect": 3},
    }
    with open(os.path.join(HERE, "sampler_golden.json"), "w") as f:
        json.dump(sampler, f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
