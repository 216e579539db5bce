"""ifr_accept_noalloc (the sampled verification with its scratch in a fixed
device array instead of a cudaMalloc'd buffer): bit-identical to ifr_accept
on two calls in a row, no change of the device's free memory across those
calls, and a clear error above its fixed scratch size.  Calls go through the
C ABI (ctypes) directly."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _err():
    from inferno_b200._lib import load
    return load().ifr_last_error().decode()


def _case(rng, B, G, V):
    tgt = rng.normal(0, 3, (B, G + 1, V)).astype(np.float32)
    dft = (tgt[:, :G] + rng.normal(0, 1.0, (B, G, V))).astype(np.float32)
    u = rng.random((B, 2 * G + 1), dtype=np.float32)
    return tgt, dft, u


def _outputs(B, G):
    import torch
    return (torch.full((B,), -7, dtype=torch.int32, device="cuda"),
            torch.full((B, G + 1), -7, dtype=torch.int32, device="cuda"),
            torch.full((B, G), -7, dtype=torch.int32, device="cuda"))


def _call(lib, fn, ctx, dev, B, G, V, T, outs=None):
    acc, out, dout = outs if outs is not None else _outputs(B, G)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = getattr(lib, fn)(ctx.handle, p(dev[0]), p(dev[1]), None, p(dev[2]), B, G, V, ctypes.c_float(T),
                          p(acc), p(out), p(dout))
    return rc, (acc, out, dout)


def test_accept_noalloc_matches_ifr_accept(pkg, ctx):
    import torch
    from inferno_b200._lib import load
    lib = load()
    rng = np.random.default_rng(2024)
    shapes = [(4, 5, 151936, 0.8), (16, 4, 32000, 1.3)]
    cases = []
    for B, G, V, T in shapes:
        dev = [torch.from_numpy(a).cuda() for a in _case(rng, B, G, V)]
        cases.append((dev, B, G, V, T))
    # one-time set-up of the fixed scratch on this device (first call)
    dev, B, G, V, T = cases[0]
    assert _call(lib, "ifr_accept_noalloc", ctx, dev, B, G, V, T)[0] == 0, _err()
    # the existing entry point (allocates the context's scratch)
    ref = []
    for dev, B, G, V, T in cases:
        rc, r = _call(lib, "ifr_accept", ctx, dev, B, G, V, T)
        assert rc == 0, _err()
        ref.append(r)
    outs = [_outputs(B, G) for _, B, G, _, _ in cases]
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    got = []
    for (dev, B, G, V, T), o in zip(cases, outs):  # two calls in a row, no sync between
        rc, r = _call(lib, "ifr_accept_noalloc", ctx, dev, B, G, V, T, o)
        assert rc == 0, _err()
        got.append(r)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    for g, r in zip(got, ref):
        for a, b, name in zip(g, r, ("accept_count", "out_tokens", "draft_tokens")):
            assert torch.equal(a, b), name


def test_accept_noalloc_rejects_oversize(pkg, ctx):
    import torch
    from inferno_b200._lib import IFR_ERR_ARG, load
    B, G, V = 128, 8, 151936  # 2*128*17*75 floats of chunk statistics > 1 MiB
    dev = [torch.zeros(1, device="cuda")] * 3
    rc, _ = _call(load(), "ifr_accept_noalloc", ctx, dev, B, G, V, 1.0)
    assert rc == IFR_ERR_ARG
    assert "scratch" in _err() and "ifr_accept" in _err()


def _torch_case(B, G, V, seed, device="cuda"):
    import torch
    gen = torch.Generator(device=device).manual_seed(seed)
    tgt = torch.randn(B, G + 1, V, generator=gen, device=device) * 3
    dft = tgt[:, :G] + torch.randn(B, G, V, generator=gen, device=device)
    u = torch.rand(B, 2 * G + 1, generator=gen, device=device)
    return [tgt.contiguous(), dft.contiguous(), u]


def test_accept_noalloc_at_scratch_limit(pkg, ctx):
    """batch 341, gamma 5, vocab 65536 needs exactly the 1 MiB of fixed
    scratch: accepted and identical to ifr_accept; one more sequence is above
    the limit and rejected"""
    import torch
    from inferno_b200._lib import IFR_ERR_ARG, load
    lib = load()
    B, G, V = 341, 5, 65536
    dev = _torch_case(B, G, V, 5)
    rc, ref = _call(lib, "ifr_accept", ctx, dev, B, G, V, 0.8)
    assert rc == 0, _err()
    rc, got = _call(lib, "ifr_accept_noalloc", ctx, dev, B, G, V, 0.8)
    assert rc == 0, _err()
    torch.cuda.synchronize()
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    del dev
    rc, _ = _call(lib, "ifr_accept_noalloc", ctx, [torch.zeros(1, device="cuda")] * 3, B + 1, G, V, 0.8)
    assert rc == IFR_ERR_ARG and "scratch" in _err()


def test_accept_noalloc_other_device(pkg):
    """a context on device 1 while device 0 is current: the one-time set-up
    looks the array up on device 1, and results match ifr_accept there"""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from inferno_b200._lib import load
    lib = load()
    torch.cuda.set_device(0)
    c1 = pkg.Context(1)
    B, G, V = 8, 4, 151936
    dev = _torch_case(B, G, V, 9, device="cuda:1")
    with torch.cuda.device(1):
        outs_ref = tuple(t.to("cuda:1") for t in _outputs(B, G))
        outs_got = tuple(t.to("cuda:1") for t in _outputs(B, G))
    assert torch.cuda.current_device() == 0
    rc, ref = _call(lib, "ifr_accept", c1, dev, B, G, V, 1.1, outs_ref)
    assert rc == 0, _err()
    rc, got = _call(lib, "ifr_accept_noalloc", c1, dev, B, G, V, 1.1, outs_got)
    assert rc == 0, _err()
    assert torch.cuda.current_device() == 0
    torch.cuda.synchronize(1)
    for a, b in zip(got, ref):
        assert torch.equal(a, b)
    c1.close()
