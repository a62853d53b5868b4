"""The NumPy-semantics oracle (oracle/newops.py) against an independent CPU implementation.

The reference has no kernel and no test for the broadcast binary ops, the unary
ops, axis reductions or the fused softmax + cross-entropy; its CPU arithmetic is
NumPy.  Here each oracle function is checked against torch on the CPU (its own
ufuncs, reductions and autograd in float64), on ragged and N-d broadcast shapes
and on NaN, +-inf, -0.0 and subnormal inputs:

* binary ops: bit-exact (IEEE add/sub/mul/div/max are correctly rounded in both);
* broadcast gradients: float64 autograd, rel 1e-12 (no ties: torch splits a tie
  of maximum/minimum, the oracle gives it to `a`, NumPy's `a >= b` choice);
* reductions: sums/means within 1 ulp of the float64 result rounded, max/min and
  arg indices exact (first index wins, NaN counts as the extreme);
* unary ops and softmax-CE: float64 evaluations rounded to float32, <= 1 ulp apart.
"""
import zlib

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import newops as O

F32 = np.float32

SHAPES = [((8, 16), (1, 16)), ((8, 16), (8, 1)), ((3, 1, 5), (1, 4, 5)), ((2, 3, 1, 4), (3, 5, 1)),
          ((7,), (1,)), ((1, 6), (5, 1)), ((0, 4), (1, 4)), ((4, 0), (4, 1)), ((), (3, 2))]


def _special(r, shape):
    x = r.standard_normal(shape).astype(F32)
    flat = x.reshape(-1)
    if flat.size >= 6:
        idx = r.choice(flat.size, min(flat.size, 6), replace=False)
        vals = np.array([np.nan, np.inf, -np.inf, -0.0, 1e-40, -3e-39], F32)
        flat[idx] = vals[:idx.size]
    return x


def _bits_equal_nan(a, b):
    a, b = np.asarray(a, F32), np.asarray(b, F32)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    return np.array_equal(na, nb) and np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))


TORCH_BINARY = {"add": torch.add, "sub": torch.sub, "mul": torch.mul, "div": torch.div,
                "maximum": torch.maximum, "minimum": torch.minimum}


@pytest.mark.parametrize("op", O.BINARY_OPS)
@pytest.mark.parametrize("shapes", SHAPES)
def test_binary_bits_match_torch(op, shapes):
    r = np.random.default_rng(zlib.crc32(repr((op, shapes)).encode()))
    a, b = _special(r, shapes[0]), _special(r, shapes[1])
    got = O.binary(op, a, b)
    want = TORCH_BINARY[op](torch.from_numpy(a), torch.from_numpy(b)).numpy()
    assert got.shape == np.broadcast_shapes(a.shape, b.shape)
    assert _bits_equal_nan(got, want)
    # and operand order swapped (right-aligned broadcasting works either way round)
    assert _bits_equal_nan(O.binary(op, b, a), TORCH_BINARY[op](torch.from_numpy(b), torch.from_numpy(a)).numpy())


@pytest.mark.parametrize("op", O.BINARY_OPS)
@pytest.mark.parametrize("shapes", [s for s in SHAPES if 0 not in s[0] + s[1] and s[0] != ()])
def test_binary_grads_match_autograd(op, shapes):
    r = np.random.default_rng(7 + O.BINARY_OPS.index(op))
    a = r.standard_normal(shapes[0]).astype(F32)
    b = (r.standard_normal(shapes[1]) + (3.0 if op == "div" else 0.0)).astype(F32)
    out_shape = np.broadcast_shapes(a.shape, b.shape)
    g = r.standard_normal(out_shape).astype(F32)
    ta = torch.tensor(a, dtype=torch.float64, requires_grad=True)
    tb = torch.tensor(b, dtype=torch.float64, requires_grad=True)
    TORCH_BINARY[op](ta, tb).backward(torch.tensor(g, dtype=torch.float64))
    ga, gb = O.binary_grads(op, a, b, g)
    assert ga.shape == a.shape and gb.shape == b.shape
    np.testing.assert_allclose(ga, ta.grad.numpy(), rtol=1e-12, atol=1e-300)
    np.testing.assert_allclose(gb, tb.grad.numpy(), rtol=1e-12, atol=1e-300)


def test_maximum_grad_tie_and_nan_rule():
    """Ties and NaN send the whole gradient to `a` (NumPy's `a >= b` pick)."""
    a = np.array([[1.0, 2.0, np.nan, 0.0]], F32)
    b = np.array([[1.0, 3.0, 5.0, np.nan]], F32)
    g = np.array([[1.0, 1.0, 1.0, 1.0]], F32)
    ga, gb = O.binary_grads("maximum", a, b, g)
    assert ga.tolist() == [[1.0, 0.0, 1.0, 0.0]] and gb.tolist() == [[0.0, 1.0, 0.0, 1.0]]
    ga, gb = O.binary_grads("minimum", a, b, g)
    assert ga.tolist() == [[1.0, 1.0, 1.0, 0.0]] and gb.tolist() == [[0.0, 0.0, 0.0, 1.0]]


@pytest.mark.parametrize("axis", [0, 1, -1, None])
@pytest.mark.parametrize("nan", [False, True])
def test_reductions_match_torch(axis, nan):
    r = np.random.default_rng(11 + (axis if axis is not None else 5) + 10 * nan)
    x = r.standard_normal((37, 53)).astype(F32)
    x[r.integers(0, 37, 20), r.integers(0, 53, 20)] = F32(1e4)       # the C3 outliers: ties in max
    if nan:
        x[3, 7] = x[20, 7] = x[5, 40] = np.nan
    tx = torch.from_numpy(x)
    kw = {} if axis is None else {"dim": axis}
    for op in ("sum", "mean"):
        got = O.reduce(op, x, axis)
        t64 = getattr(torch, op)(tx.double(), **kw).numpy().astype(F32)
        assert np.asarray(got).shape == np.asarray(t64).shape
        nm = np.isnan(t64)
        assert np.array_equal(np.isnan(got), nm)
        assert O.ulp_diff(np.asarray(got)[~nm], np.asarray(t64)[~nm]).max(initial=0) <= 1, op
    for op, fn in (("max", torch.amax), ("min", torch.amin)):
        got = O.reduce(op, x, axis)
        want = (fn(tx) if axis is None else fn(tx, dim=axis)).numpy()
        assert _bits_equal_nan(got, want), op
    for op, fn in (("argmax", torch.argmax), ("argmin", torch.argmin)):
        got = O.reduce(op, x, axis)
        want = (fn(tx) if axis is None else fn(tx, dim=axis)).numpy()
        assert np.array_equal(np.asarray(got, np.int64), want), op


def test_argmax_first_index_and_nan_wins():
    x = np.array([[1, 5, 5, 2], [np.nan, 9, np.nan, 9], [-np.inf, -np.inf, -np.inf, -np.inf]], F32)
    assert O.reduce("argmax", x, 1).tolist() == [1, 0, 0]
    assert O.reduce("argmin", x, 1).tolist() == [0, 0, 0]
    assert O.reduce("argmax", x.T, 0).tolist() == [1, 0, 0]


@pytest.mark.parametrize("op,fn", [("exp", torch.exp), ("tanh", torch.tanh), ("sigmoid", torch.sigmoid),
                                   ("log_abs1p", None)])
def test_unary_reference_matches_torch_f64(op, fn):
    r = np.random.default_rng(21)
    x = np.concatenate([(6 * r.standard_normal(20000)).astype(F32),
                        np.array([0.0, -0.0, 88.7, -103.9, 1e-40, -1e-40, np.inf, -np.inf, np.nan], F32)])
    got = O.unary_f64(op, x)
    if fn is None:
        t = torch.from_numpy((np.abs(x) + F32(1.0)).astype(F32)).double()
        want = torch.log(t).numpy().astype(F32)
    else:
        want = fn(torch.from_numpy(x).double()).numpy().astype(F32)
    nm = np.isnan(want)
    assert np.array_equal(np.isnan(got), nm)
    assert O.ulp_diff(got[~nm], want[~nm]).max() <= 1


@pytest.mark.parametrize("B,K", [(64, 1000), (5, 3), (1, 1), (33, 257)])
def test_softmax_ce_matches_torch(B, K):
    r = np.random.default_rng(B * 1000 + K)
    logits = (3 * r.standard_normal((B, K))).astype(F32)
    labels = r.integers(0, K, B)
    p, loss, logp = O.softmax_ce_f64(logits, labels)
    t = torch.tensor(logits, dtype=torch.float64, requires_grad=True)
    tl = torch.nn.functional.cross_entropy(t, torch.from_numpy(labels), reduction="mean")
    tl.backward()
    assert O.ulp_diff(p, torch.softmax(t, 1).detach().numpy().astype(F32)).max() <= 1
    assert O.ulp_diff(logp, torch.log_softmax(t, 1).detach().numpy().astype(F32)).max() <= 1
    assert O.ulp_diff(np.array([loss], F32), np.array([tl.item()], F32)).max() <= 1
    # dlogits from the oracle's probs against autograd's float64 gradient
    d = O.softmax_ce_dlogits(p, labels, B)
    np.testing.assert_allclose(d, t.grad.numpy(), rtol=1e-6, atol=1e-7 / B)
    # sharded rows: a global divisor gives each shard's share of the mean
    if B > 2:
        h = B // 2
        _, l1, _ = O.softmax_ce_f64(logits[:h], labels[:h], loss_divisor=B)
        _, l2, _ = O.softmax_ce_f64(logits[h:], labels[h:], loss_divisor=B)
        np.testing.assert_allclose(float(l1) + float(l2), tl.item(), rtol=1e-6)


def test_ulp_diff_known_answers():
    one = np.array([1.0], F32)
    assert O.ulp_diff(one, np.nextafter(one, F32(2))).tolist() == [1]
    assert O.ulp_diff(np.array([0.0], F32), np.array([-0.0], F32)).tolist() == [0]
    tiny = np.array([1e-45], F32)                                   # the smallest subnormal
    assert O.ulp_diff(tiny, -tiny).tolist() == [2]
    assert O.ulp_diff(np.array([np.inf], F32), np.array([np.finfo(F32).max], F32)).tolist() == [1]


def test_empty_operands():
    """Empty operands: NumPy's sum 0 / mean NaN / extremes raise, and the reference
    loss over an empty batch is 0/0 = NaN (nn_loss.hlsl:41) in the shader oracle."""
    import warnings
    from oracle import shaders as S
    e = np.zeros((3, 0, 4), F32)
    assert np.array_equal(O.reduce("sum", e, 1), np.zeros((3, 4), F32))
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", RuntimeWarning)
        assert np.isnan(O.reduce("mean", e, 1)).all()
        assert np.isnan(S.ce_loss_f64(np.zeros(4, F32), np.zeros(1, F32), 0, 4))
    for op in ("max", "argmax", "min", "argmin"):
        with pytest.raises(ValueError):
            O.reduce(op, e, 1)
    assert O.binary("add", np.zeros((0, 4), F32), np.ones((1, 4), F32)).shape == (0, 4)
