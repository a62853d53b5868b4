"""The allocation-free BatchNorm training forward, checked against the ordinary one.

`dct_batchnorm_forward_train_noalloc` is for callers that cannot let the
library allocate device memory (their HBM already belongs to their own
allocator, or they run to a fixed memory budget): it takes caller-owned device
pointers and keeps its float64 partial sums in a fixed device array instead of
the library's growable workspace.  Here it runs twice in a row -- the second
call sees the first call's leftovers in that shared array -- and each time its
y, batch mean / variance and running statistics must match
`dct_batchnorm_forward_train` on identical inputs, within the tolerances of
the BatchNorm tests (statistics rel 1e-6, y bit-exact given the statistics).
This file is collected last so a run that stops at the first failure has run
every other test already; it also passes alone in a fresh process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ptr(dev, h):
    return dev.lib.dct_buffer_device_ptr(h)


def _stream(dev, kind):
    """The stream a caller would pass: the library's own, one the caller created
    (a PyTorch stream), or 0 (the legacy default stream)."""
    if kind == "library":
        return dev.lib.dct_stream(), None
    if kind == "null":
        return None, None
    torch = pytest.importorskip("torch")
    s = torch.cuda.Stream(device=dev.lib.dct_device())
    return s.cuda_stream, s


def _wait(dev, kind, tstream):
    """Make the allocation-free call's work visible to the library's reads."""
    if kind == "library":
        return
    import torch
    if tstream is not None:
        tstream.synchronize()
    else:
        torch.cuda.synchronize(dev.lib.dct_device())


@pytest.mark.parametrize("stream_kind", ["library", "caller", "null"])
@pytest.mark.parametrize("shape", [(4, 16, 7, 7), (32, 256, 28, 28)])
def test_noalloc_matches_allocating_entry_point_twice(dev, shape, stream_kind):
    N, C, H, W = shape
    S = H * W
    lib = dev.lib
    r = np.random.default_rng(20)
    x = (0.5 + 2 * r.standard_normal(shape)).astype(np.float32)
    gamma = r.random(C, dtype=np.float32)
    beta = r.random(C, dtype=np.float32)
    rm0 = (0.1 * r.standard_normal(C)).astype(np.float32)
    rv0 = (1.0 + r.random(C, dtype=np.float32)).astype(np.float32)
    hx, hg, hb = dev.buf(x), dev.buf(gamma), dev.buf(beta)
    # the ordinary entry point's outputs
    a_rm, a_rv, a_m, a_v, a_y = dev.buf(rm0), dev.buf(rv0), dev.empty(C), dev.empty(C), dev.empty(x.size)
    # the allocation-free entry point's outputs (same initial running statistics)
    b_rm, b_rv, b_m, b_v, b_y = dev.buf(rm0), dev.buf(rv0), dev.empty(C), dev.empty(C), dev.empty(x.size)
    stream, tstream = _stream(dev, stream_kind)
    for call in range(2):
        rc = lib.dct_batchnorm_forward_train(hx, hg, hb, a_rm, a_rv, a_m, a_v, a_y, N, C, S, 1e-5, 0.1)
        assert rc == 0, dev.error()
        dev.sync()                             # inputs ready before another stream reads them
        rc = lib.dct_batchnorm_forward_train_noalloc(
            _ptr(dev, hx), _ptr(dev, hg), _ptr(dev, hb), _ptr(dev, b_rm), _ptr(dev, b_rv), _ptr(dev, b_m),
            _ptr(dev, b_v), _ptr(dev, b_y), N, C, S, 1e-5, 0.1, stream)
        assert rc == 0, dev.error()
        _wait(dev, stream_kind, tstream)
        for name, ha, hb_ in (("mean", a_m, b_m), ("var", a_v, b_v), ("running_mean", a_rm, b_rm),
                              ("running_var", a_rv, b_rv)):
            want, got = dev.read(ha), dev.read(hb_)
            assert np.allclose(got, want, rtol=1e-6, atol=1e-8), (call, name, np.abs(got - want).max())
        ya, yb = dev.read(a_y), dev.read(b_y)
        if np.array_equal(dev.read(a_m), dev.read(b_m)) and np.array_equal(dev.read(a_v), dev.read(b_v)):
            assert np.array_equal(yb.view(np.uint32), ya.view(np.uint32)), call
        else:
            assert np.allclose(yb, ya, rtol=1e-5, atol=1e-6), call
    dev.free(hx, hg, hb, a_rm, a_rv, a_m, a_v, a_y, b_rm, b_rv, b_m, b_v, b_y)


def test_noalloc_rejects_shapes_beyond_its_scratch(dev):
    lib = dev.lib
    h = dev.empty(16, fill=7.0)
    p = _ptr(dev, h)
    dev.clear_error()
    # 2 x 65537 = 131074 planes > 131072
    rc = lib.dct_batchnorm_forward_train_noalloc(p, p, p, p, p, p, p, p, 2, 65537, 1, 1e-5, 0.1, lib.dct_stream())
    assert rc == 3
    code, msg = dev.error()
    assert code == 3 and "131072" in msg
    rc = lib.dct_batchnorm_forward_train_noalloc(p, p, p, p, p, p, p, p, 1, 4097, 1, 1e-5, 0.1, lib.dct_stream())
    assert rc == 3
    assert (dev.read(h) == 7.0).all()       # nothing was launched
    dev.free(h)


@pytest.mark.parametrize("empty", [(0, 8, 5, 5), (3, 8, 0, 4)], ids=["N=0", "S=0"])
def test_noalloc_empty_batch_matches_allocating_entry_point(dev, empty):
    """A batch with no elements: both entry points compute statistics over nothing
    (0 / 0) and update the running statistics the same way."""
    N, C, H, W = empty
    S = H * W
    lib = dev.lib
    x = dev.empty(16)
    g, b = dev.buf(np.ones(C, np.float32)), dev.buf(np.zeros(C, np.float32))
    rm0, rv0 = np.full(C, 0.25, np.float32), np.full(C, 2.0, np.float32)
    outs = []
    for noalloc in (False, True):
        rm, rv, m, v, y = dev.buf(rm0), dev.buf(rv0), dev.empty(C), dev.empty(C), dev.empty(16)
        if noalloc:
            rc = lib.dct_batchnorm_forward_train_noalloc(_ptr(dev, x), _ptr(dev, g), _ptr(dev, b), _ptr(dev, rm),
                                                         _ptr(dev, rv), _ptr(dev, m), _ptr(dev, v), _ptr(dev, y),
                                                         N, C, S, 1e-5, 0.1, lib.dct_stream())
        else:
            rc = lib.dct_batchnorm_forward_train(x, g, b, rm, rv, m, v, y, N, C, S, 1e-5, 0.1)
        assert rc == 0, dev.error()
        dev.sync()
        outs.append([dev.read(h) for h in (rm, rv, m, v)])
        dev.free(rm, rv, m, v, y)
    for a, c in zip(*outs):
        assert np.array_equal(a.view(np.uint32), c.view(np.uint32)) or (np.isnan(a).all() and np.isnan(c).all())
    dev.free(x, g, b)
