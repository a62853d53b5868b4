"""NumPy-semantics ops (no reference kernel) through the dct_* C-ABI vs the oracle.

Broadcast binary ops: bit-exact vs NumPy float32.  Unary exp/log(|x|+1)/tanh/
sigmoid: <= 2 ulp vs float64 rounded.  Sums/means: rel 1e-5 vs float64
accumulation (measured much tighter).  max/argmax: exact (first index, NaN wins).
"""
import zlib

import numpy as np
import pytest

from oracle import newops as O

pytestmark = pytest.mark.gpu


def _same(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    assert a.shape == b.shape, (a.shape, b.shape)
    eq = (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
    if not eq.all():
        i = np.flatnonzero(~eq.ravel())[:5]
        raise AssertionError(f"{(~eq).sum()} mismatches at {i}: got {a.ravel()[i]} want {b.ravel()[i]}")


BCAST_CASES = [
    ((7,), (7,)),
    ((5, 8), (8,)),
    ((5, 8), (1, 8)),
    ((8,), (5, 8)),
    ((6, 1), (6, 7)),
    ((3, 1, 5), (1, 4, 5)),
    ((2, 3, 4, 5), (3, 1, 5)),
    ((4, 1, 3, 1), (1, 5, 1, 6)),
    ((1,), (9, 13)),
    ((9, 13), ()),
    ((2, 1, 3, 1, 2, 1, 2, 1), (1, 2, 1, 3, 1, 2, 1, 2)),
    ((64, 1, 1024), (1, 128, 1024)),
    ((257, 1023), (1023,)),
    ((16, 1, 12), (16, 33, 12)),
]


@pytest.mark.parametrize("op", O.BINARY_OPS)
@pytest.mark.parametrize("shapes", BCAST_CASES)
def test_binary_broadcast_bitexact(dev, op, shapes):
    sa, sb = shapes
    r = np.random.default_rng(zlib.crc32(repr((op, shapes)).encode()))
    a = r.standard_normal(sa).astype(np.float32)
    b = (r.random(sb) * 1.5 + 0.5).astype(np.float32)
    if a.size > 8:
        a.flat[:4] = [np.nan, np.inf, -0.0, 0.0]
    want = O.binary(op, a, b)
    ha, hb, ho = dev.buf(a), dev.buf(np.atleast_1d(b)), dev.empty(want.size)
    dev.binary(op, ha, list(sa), hb, list(sb), ho)
    _same(dev.read(ho).reshape(want.shape), want)
    dev.free(ha, hb, ho)


def test_binary_shape_mismatch_is_an_error(dev):
    ha, hb, ho = dev.empty(6), dev.empty(4), dev.empty(24)
    with pytest.raises(RuntimeError, match="ARG"):
        dev.binary("add", ha, [2, 3], hb, [4], ho)
    dev.free(ha, hb, ho)


@pytest.mark.parametrize("op", ["exp", "log_abs1p", "tanh", "sigmoid"])
@pytest.mark.parametrize("n", [1, 5, 1000, 1 << 20])
def test_unary_2ulp(dev, op, n):
    r = np.random.default_rng(n)
    x = (r.standard_normal(n) * 4).astype(np.float32)
    if n > 16:
        x[:10] = [0.0, -0.0, np.inf, -np.inf, np.nan, 88.0, -88.0, 1e-30, -103.0, 20.0]
    want = O.unary_f64(op, x)
    hx, hy = dev.buf(x), dev.empty(n)
    dev.unary(op, hx, hy, n)
    got = dev.read(hy)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    u = O.ulp_diff(got[~nan], want[~nan])
    assert u.max() <= 2, f"max ulp {u.max()} at x={x[~nan][u.argmax()]}"
    dev.free(hx, hy)


def test_sigmoid_whole_range(dev):
    """Every binade of the float range, 5M dense samples in [-20, 20], the
    subnormal-result tail (-87.3 > x > -104), +-inf, NaN and signed zeros: <= 2 ulp
    against the float64 result rounded (the result's subnormal spacing counts as its
    ulp)."""
    r = np.random.default_rng(77)
    parts = [np.float32(2.0) ** np.arange(-149, 128, dtype=np.float64).astype(np.float32)]
    parts.append(r.uniform(-110, -80, 1 << 18).astype(np.float32))
    parts.append(r.uniform(80, 110, 1 << 12).astype(np.float32))
    parts.append(r.uniform(-20, 20, 1 << 22).astype(np.float32))        # dense where sigmoid is not 0 / 1
    parts.append((3 * r.standard_normal(1 << 20)).astype(np.float32))
    parts.append(np.array([0.0, -0.0, np.inf, -np.inf, np.nan, -87.33655, -103.97, -104.0, 104.0, -1e30, 3e38],
                          np.float32))
    x = np.concatenate([parts[0], -parts[0]] + parts[1:]).astype(np.float32)
    with np.errstate(all="ignore"):
        want = (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)
    hx, hy = dev.buf(x), dev.empty(x.size)
    dev.unary("sigmoid", hx, hy, x.size)
    got = dev.read(hy)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    d = np.abs(got[~nan].view(np.int32).astype(np.int64) - want[~nan].view(np.int32).astype(np.int64))
    assert d.max() <= 2, f"max ulp {d.max()} at x={x[~nan][d.argmax()]}"
    assert got[x == np.inf][0] == 1.0 and got[x == -np.inf][0] == 0.0
    dev.free(hx, hy)


def _assert_rel_1e5(got, want64, mag, what):
    """|got - want| <= 1e-5 |want| (a true relative bound on the float64-accumulated
    result) + 1e-12 * sum|x| (the float64 accumulation's own order-dependent noise,
    relevant only where the terms cancel to almost nothing)."""
    got, want64, mag = (np.asarray(a, np.float64) for a in (got, want64, mag))
    err = np.abs(got - want64)
    bound = 1e-5 * np.abs(want64) + 1e-12 * mag
    assert np.all(err <= bound), (what, float((err / np.maximum(bound, 1e-300)).max()))


def _rel(got, want64):
    want64 = np.asarray(want64, np.float64)
    return np.abs(got.astype(np.float64) - want64) / np.maximum(np.abs(want64), 1e-30)


def _R(rows, cols, seed):
    r = np.random.default_rng(seed)
    x = r.standard_normal((rows, cols)).astype(np.float32)
    k = max(1, x.size // 1000)
    idx = r.choice(x.size, k, replace=False)
    x.flat[idx] = np.where(r.integers(0, 2, k) == 1, 1e4, -1e4).astype(np.float32)
    return x


@pytest.mark.parametrize("shape", [(1, 1), (3, 5), (17, 4097), (1024, 4096), (5, 300000), (4096, 3)])
@pytest.mark.parametrize("axis", [0, 1])
def test_axis_reductions(dev, shape, axis):
    x = _R(*shape, seed=sum(shape) + axis)
    rows, cols = shape
    outer, length, inner = (1, rows, cols) if axis == 0 else (rows, cols, 1)
    nout = outer * inner
    hx = dev.buf(x)
    ho, hi = dev.empty(nout), dev.empty(nout)
    x64 = x.astype(np.float64)
    for op in ("sum", "mean"):
        dev.reduce(op, hx, outer, length, inner, ho)
        want = x64.sum(axis=axis) if op == "sum" else x64.mean(axis=axis)
        got = dev.read(ho)
        mag = np.abs(x64).sum(axis=axis) / (1 if op == "sum" else x64.shape[axis])
        _assert_rel_1e5(got, want, mag, op)
    dev.reduce("max", hx, outer, length, inner, ho, hi)
    _same(dev.read(ho), x.max(axis=axis))
    assert np.array_equal(dev.read(hi, np.int32), x.argmax(axis=axis))
    dev.reduce("argmax", hx, outer, length, inner, hi)
    assert np.array_equal(dev.read(hi, np.int32), x.argmax(axis=axis))
    dev.reduce("argmin", hx, outer, length, inner, hi)
    assert np.array_equal(dev.read(hi, np.int32), x.argmin(axis=axis))
    dev.free(hx, ho, hi)


def test_argmax_ties_and_nan(dev):
    x = np.array([[1, 3, 3, 2], [np.nan, 1, np.nan, 5], [2, 2, 2, 2], [-np.inf, -np.inf, -1, -1]], np.float32)
    hx, ho, hi = dev.buf(x), dev.empty(4), dev.empty(4)
    dev.reduce("max", hx, 4, 4, 1, ho, hi)
    assert np.array_equal(dev.read(hi, np.int32), np.argmax(x, axis=1))
    got = dev.read(ho)
    assert np.isnan(got[1]) and got[0] == 3 and got[2] == 2 and got[3] == -1
    dev.reduce("max", hx, 1, 4, 4, ho, hi)
    assert np.array_equal(dev.read(hi, np.int32), np.argmax(x, axis=0))
    dev.free(hx, ho, hi)


@pytest.mark.parametrize("n", [1, 7, 4096, 1 << 22, (1 << 22) + 3])
def test_full_sum(dev, n):
    r = np.random.default_rng(n)
    x = (r.random(n, dtype=np.float32) * 2 - 1).astype(np.float32)
    hx, ho = dev.buf(x), dev.empty(1)
    v64 = dev.reduce_all("sum", hx, n, ho)
    ref = O.full_sum_f64(x)
    assert abs(v64 - ref) <= 1e-9 * max(1.0, np.abs(x).sum())
    assert dev.read(ho)[0] == np.float32(v64)
    m = dev.reduce_all("max", hx, n, ho)
    assert np.float32(m) == x.max()
    dev.free(hx, ho)


@pytest.mark.parametrize("BK", [(1, 1), (7, 10), (64, 1000), (33, 1001), (512, 128), (16, 2048), (8, 5000)])
@pytest.mark.parametrize("int_labels", [False, True])
def test_fused_softmax_ce(dev, BK, int_labels):
    B, K = BK
    r = np.random.default_rng(B * 7 + K)
    x = (3 * r.standard_normal((B, K))).astype(np.float32)
    lab = r.integers(0, K, B)
    p_ref, loss_ref, lp_ref = O.softmax_ce_f64(x, lab)
    hx = dev.buf(x)
    hl = dev.buf(lab.astype(np.int32) if int_labels else lab.astype(np.float32))
    hp, hg, hloss, hlp = dev.empty(B * K), dev.empty(B * K), dev.empty(1), dev.empty(B * K)
    lib = dev.lib
    rc = lib.dct_softmax_ce(hx, hl, int(int_labels), B, K, hp, hg, hloss, hlp, float(B), float(B))
    assert rc == 0, dev.error()
    p = dev.read(hp).reshape(B, K)
    u = O.ulp_diff(p, p_ref)
    assert u.max() <= 4, u.max()
    assert np.abs(dev.read(hloss)[0] - loss_ref) <= 1e-6 * max(1.0, abs(loss_ref))
    _same(dev.read(hg).reshape(B, K), O.softmax_ce_dlogits(p, lab, B))
    lp = dev.read(hlp).reshape(B, K)
    assert O.ulp_diff(lp, lp_ref).max() <= 2
    dev.free(hx, hl, hp, hg, hloss, hlp)


def test_adam_bitexact(dev):
    from oracle import shaders as S
    r = np.random.default_rng(4)
    n = 1000003
    w = (r.standard_normal(n) * 0.02).astype(np.float32)
    g = (r.standard_normal(n) * 1e-3).astype(np.float32)
    g[:3] = [5.0, -5.0, np.nan]
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    hw, hm, hv, hg = dev.buf(w), dev.buf(m), dev.buf(v), dev.buf(g)
    for t in range(1, 4):
        step = S.adam_step_size(1e-3, 0.9, 0.999, t)
        rc = dev.lib.dct_adam(hw, hm, hv, hg, n, float(step), 0.9, 0.999, 1e-8, 0.0, 1.0)
        assert rc == 0
        w, m, v = S.adam(w, m, v, g, n, step, 0.9, 0.999, 1e-8, 0.0, 1.0)
    _same(dev.read(hw), w)
    _same(dev.read(hm), m)
    _same(dev.read(hv), v)
    dev.free(hw, hm, hv, hg)


@pytest.mark.parametrize("shape", [(6, 40, 512), (3, 1000, 4096), (2, 9, 8192), (5, 64, 12)])
def test_middle_axis_reductions(dev, shape):
    """[outer, len, inner] reduced over the middle axis (column kernels with outer > 1)."""
    P, L, Q = shape
    x = _R(P * L, Q, seed=P + L + Q).reshape(P, L, Q)
    hx = dev.buf(x)
    ho, hi = dev.empty(P * Q), dev.empty(P * Q)
    x64 = x.astype(np.float64)
    dev.reduce("sum", hx, P, L, Q, ho)
    want = x64.sum(axis=1).ravel()
    _assert_rel_1e5(dev.read(ho), want, np.abs(x64).sum(axis=1).ravel(), "middle-axis sum")
    dev.reduce("argmax", hx, P, L, Q, hi)
    assert np.array_equal(dev.read(hi, np.int32), x.argmax(axis=1).ravel())
    dev.reduce("min", hx, P, L, Q, ho)
    _same(dev.read(ho), x.min(axis=1).ravel())
    dev.free(hx, ho, hi)
