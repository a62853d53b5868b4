"""Broadcast gradients and the autograd ops of `directcompute_torch_b200.ops`.

`dct_sum_to_shape` (the broadcast gradient) against the float64 oracle
`newops.sum_to_shape` over every collapse pattern: one reduced group (row,
column and middle-axis kernels) and several (the generic kernel, chunked and
not).  The ops' forward values are bit-exact against NumPy float32 (binary
ops) or within 2 ulp of float64 (transcendentals); gradients are within
rel 1e-5 of the float64 oracle `newops.binary_grads` (the device rounds each
elementwise factor to float32 before the float64 sum).
"""
import ctypes

import numpy as np
import pytest

from oracle import newops as O

pytestmark = pytest.mark.gpu

STS_CASES = [
    ((7,), (7,)),                     # nothing reduced: copy
    ((5, 8), (8,)),                   # leading dim: column kernel
    ((5, 8), (5, 1)),                 # trailing dim: row kernel
    ((6, 40, 512), (6, 1, 512)),      # middle axis
    ((3, 1000, 4096), (1, 1, 4096)),  # leading dims merged
    ((4, 5, 3, 6), (4, 1, 3, 1)),     # two reduced groups: generic
    ((9, 7, 11), (1, 7, 1)),          # [R, K, R]
    ((2, 3, 4, 5, 6), (3, 1, 5, 1)),  # [R, K, R, K, R]
    ((64, 512, 4096), (64, 1, 4096)), # C2 outer-broadcast operand C
    ((64, 512, 4096), (512, 4096)),   # and D
    ((8192, 8192), (1, 8192)),        # C2 row-broadcast operand B
    ((3, 5), ()),                     # to a scalar
    ((1, 5, 1), (5, 1)),              # size-1 dims in g
]


def _sts(dev, g, t_shape):
    lib = dev.lib
    hg = dev.buf(g)
    n = int(np.prod(t_shape)) if len(t_shape) else 1
    ho = dev.empty(n)
    G = (ctypes.c_int64 * max(1, g.ndim))(*g.shape)
    T = (ctypes.c_int64 * max(1, len(t_shape)))(*t_shape)
    assert lib.dct_sum_to_shape(hg, G, g.ndim, T, len(t_shape), ho) == 0, dev.error()
    out = dev.read(ho)[:n].reshape(t_shape)
    dev.free(hg, ho)
    return out


@pytest.mark.parametrize("shapes", STS_CASES)
def test_sum_to_shape_matches_oracle(dev, shapes):
    g_shape, t_shape = shapes
    r = np.random.default_rng(50)
    g = r.standard_normal(g_shape).astype(np.float32)
    got = _sts(dev, g, t_shape)
    want = O.sum_to_shape(g, t_shape)
    scale = np.sqrt(np.prod(g_shape) / max(1, np.prod(t_shape)))
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6 * scale)
    # float64 accumulation rounded once: nearly every element is the correctly rounded sum
    exact = np.mean(got == want.astype(np.float32))
    assert exact > 0.99, exact


def test_sum_to_shape_rejects_non_broadcast(dev):
    lib = dev.lib
    hg, ho = dev.empty(20), dev.empty(20)
    G = (ctypes.c_int64 * 2)(4, 5)
    T = (ctypes.c_int64 * 2)(2, 5)
    assert lib.dct_sum_to_shape(hg, G, 2, T, 2, ho) == 4          # DCT_ERR_ARG
    dev.clear_error()
    dev.free(hg, ho)


@pytest.mark.parametrize("shapes", [((1, 8), (5, 8)), ((8,), (5, 8)), ((64, 1, 32), (64, 16, 32)), ((3, 1), (3, 4)),
                                    ((1, 1), (37, 129))])
def test_broadcast_to(dev, shapes):
    x_shape, out_shape = shapes
    lib = dev.lib
    x = np.random.default_rng(51).standard_normal(x_shape).astype(np.float32)
    hx, ho = dev.buf(x), dev.empty(int(np.prod(out_shape)))
    X = (ctypes.c_int64 * len(x_shape))(*x_shape)
    S = (ctypes.c_int64 * len(out_shape))(*out_shape)
    assert lib.dct_broadcast_to(hx, X, len(x_shape), S, len(out_shape), ho) == 0, dev.error()
    np.testing.assert_array_equal(dev.read(ho).reshape(out_shape), np.broadcast_to(x, out_shape))
    dev.free(hx, ho)


# ---------------------------------------------------------------------------
# autograd ops
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def ops(dev):
    from directcompute_torch_b200 import ops as _ops
    return _ops


BIN_SHAPES = [((5, 8), (8,)), ((6, 1), (6, 7)), ((3, 1, 5), (1, 4, 5)), ((4, 1, 3, 1), (1, 5, 1, 6)),
              ((257, 1023), (257, 1023)), ((7,), ())]


@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "maximum", "minimum"])
@pytest.mark.parametrize("shapes", BIN_SHAPES)
def test_binary_forward_and_broadcast_grad(dev, ops, op, shapes):
    sa, sb = shapes
    r = np.random.default_rng(52)
    a = r.standard_normal(sa).astype(np.float32)
    b = r.standard_normal(sb).astype(np.float32)
    if op == "div":
        b = np.where(np.abs(b) < 0.1, np.float32(0.5), b).astype(np.float32)
    if op in ("maximum", "minimum") and a.size > 3:
        a.ravel()[1] = np.nan                                     # NaN in a: gradient to a
        if a.shape == b.shape:
            a.ravel()[2] = b.ravel()[2] = 0.25                    # tie: gradient to a
    A = ops.tensor(a, requires_grad=True)
    B = ops.tensor(b, requires_grad=True)
    out = getattr(ops, op)(A, B)
    want = O.binary(op, a, b)
    got = ops.to_numpy(out)
    assert got.shape == want.shape
    eq = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert eq.all(), (op, shapes)
    g = r.standard_normal(want.shape).astype(np.float32)
    out.backward(ops.tensor(g))
    ga, gb = O.binary_grads(op, a, b, g)
    for name, t, w in (("a", A, ga), ("b", B, gb)):
        got_g = ops.to_numpy(t.grad).reshape(w.shape)
        fin = np.isfinite(w)
        scale = np.sqrt(g.size / max(1, w.size))
        np.testing.assert_allclose(got_g[fin], w[fin], rtol=1e-5, atol=1e-6 * scale, err_msg=f"{op} grad {name}")


@pytest.mark.parametrize("op", ["exp", "log_abs1p", "tanh", "sigmoid", "neg", "abs"])
def test_unary_forward_and_grad(dev, ops, op):
    r = np.random.default_rng(53)
    x = (3 * r.standard_normal(4099)).astype(np.float32)
    x[:3] = (0.0, -0.0, 1e-30)
    X = ops.tensor(x, requires_grad=True)
    y = getattr(ops, op)(X)
    got = ops.to_numpy(y)
    want = O.unary_f64(op, x)
    assert O.ulp_diff(got, want).max() <= 2, op
    g = r.standard_normal(x.shape).astype(np.float32)
    y.backward(ops.tensor(g))
    x64, g64, y64 = x.astype(np.float64), g.astype(np.float64), got.astype(np.float64)
    with np.errstate(all="ignore"):
        dydx = {"exp": y64, "tanh": 1 - y64 * y64, "sigmoid": y64 * (1 - y64),
                "log_abs1p": np.sign(x64) / (np.abs(x64) + 1), "neg": -np.ones_like(x64),
                "abs": np.sign(x64)}[op]
    # each factor is rounded to float32 on the device (1 - y*y loses to cancellation near |y| = 1)
    err = np.abs(ops.to_numpy(X.grad) - g64 * dydx)
    assert np.all(err <= 2e-6 * np.abs(g64 * dydx) + 1.2e-7 * np.abs(g64)), (op, err.max())


@pytest.mark.parametrize("axis", [None, 0, 1, -1])
def test_reductions_and_their_grads(dev, ops, axis):
    r = np.random.default_rng(54)
    x = r.standard_normal((37, 129)).astype(np.float32)
    for op in ("sum", "mean", "max", "min"):
        X = ops.tensor(x, requires_grad=True)
        y = getattr(ops, op)(X, axis=axis)
        got = ops.to_numpy(y)
        want = O.reduce(op, x, axis) if axis is not None else O.reduce(op, x.ravel(), 0)
        np.testing.assert_allclose(got.reshape(np.shape(want)), want, rtol=1e-6, atol=1e-6)
        if op in ("sum", "mean"):
            g = r.standard_normal(np.shape(want) or (1,)).astype(np.float32)
            y.backward(ops.tensor(g.reshape(y.shape)))
            gx = np.broadcast_to(np.expand_dims(g.reshape(np.shape(want)), axis) if axis is not None
                                 else g.reshape(()), x.shape).astype(np.float64)
            if op == "mean":
                n = x.size if axis is None else x.shape[axis]
                gx = gx * np.float64(np.float32(1.0 / n))
            np.testing.assert_allclose(ops.to_numpy(X.grad), gx, rtol=1e-6, atol=1e-7)
    ax = axis if axis is not None else None
    am = ops.argmax(ops.tensor(x), axis=ax)
    np.testing.assert_array_equal(am, np.argmax(x, axis=ax))


def test_softmax_cross_entropy_op(dev, ops):
    r = np.random.default_rng(55)
    B, K = 300, 37
    x = (3 * r.standard_normal((B, K))).astype(np.float32)
    lab = r.integers(0, K, B)
    X = ops.tensor(x, requires_grad=True)
    loss, probs = ops.softmax_cross_entropy(X, ops.tensor(lab.astype(np.float32)), return_probs=True)
    p64, l64, _ = O.softmax_ce_f64(x, lab)
    assert abs(float(ops.to_numpy(loss)[0]) - float(l64)) <= 1e-5 * abs(float(l64))
    loss.backward(ops.tensor(np.array([2.0], np.float32)))
    want = 2.0 * O.softmax_ce_dlogits(ops.to_numpy(probs), lab, B).astype(np.float64)
    np.testing.assert_allclose(ops.to_numpy(X.grad), want, rtol=1e-6, atol=1e-9)


def test_chain_rule_through_broadcast(dev, ops):
    """loss = mean((x * w + b) ** 2 via mul), x [64, 32], w [32], b [1]."""
    r = np.random.default_rng(56)
    x = r.standard_normal((64, 32)).astype(np.float32)
    w = r.standard_normal(32).astype(np.float32)
    b = r.standard_normal(1).astype(np.float32)
    X, W, Bt = ops.tensor(x), ops.tensor(w, requires_grad=True), ops.tensor(b, requires_grad=True)
    z = ops.add(ops.mul(X, W), Bt)
    loss = ops.mean(ops.mul(z, z))
    loss.backward()
    z64 = x.astype(np.float64) * w + b
    dz = 2 * z64 / z64.size
    np.testing.assert_allclose(ops.to_numpy(W.grad), (dz * x).sum(axis=0), rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(ops.to_numpy(Bt.grad), [dz.sum()], rtol=1e-5, atol=1e-7)


# ---------------------------------------------------------------------------
# bias + ReLU and BatchNorm2d ops against PyTorch (float32 on the CPU)
# ---------------------------------------------------------------------------
def test_dense_head_bias_relu_softmax_ce_vs_torch(dev, ops):
    """softmax-CE(bias_relu(x, b)): the loss and both gradients, the backward of
    bias_relu in one fused pass (dct_bias_relu_backward)."""
    torch = pytest.importorskip("torch")
    r = np.random.default_rng(23)
    B, K = 64, 10
    x = (2 * r.standard_normal((B, K))).astype(np.float32)
    b = (0.1 * r.standard_normal(K)).astype(np.float32)
    lab = r.integers(0, K, B)
    X, Bt = ops.tensor(x, requires_grad=True), ops.tensor(b, requires_grad=True)
    h = ops.bias_relu(X, Bt)
    np.testing.assert_array_equal(ops.to_numpy(h), np.maximum(x + b, 0).astype(np.float32))
    loss = ops.softmax_cross_entropy(h, ops.tensor(lab.astype(np.float32)))
    loss.backward()
    xt = torch.tensor(x, requires_grad=True)
    bt = torch.tensor(b, requires_grad=True)
    lt = torch.nn.functional.cross_entropy(torch.relu(xt + bt), torch.tensor(lab))
    lt.backward()
    assert abs(float(ops.to_numpy(loss)[0]) - float(lt.detach())) <= 1e-5 * abs(float(lt.detach()))
    np.testing.assert_allclose(ops.to_numpy(X.grad), xt.grad.numpy(), rtol=1e-5, atol=1e-8)
    np.testing.assert_allclose(ops.to_numpy(Bt.grad), bt.grad.numpy(), rtol=1e-5, atol=1e-8)


def test_batch_norm2d_train_and_eval_vs_torch(dev, ops):
    torch = pytest.importorskip("torch")
    r = np.random.default_rng(24)
    x = (0.5 + 2 * r.standard_normal((8, 4, 6, 6))).astype(np.float32)
    g = r.standard_normal((8, 4, 6, 6)).astype(np.float32)
    gamma, beta = r.random(4, dtype=np.float32) + 0.5, r.standard_normal(4).astype(np.float32)
    X = ops.tensor(x, requires_grad=True)
    G, Be = ops.tensor(gamma, requires_grad=True), ops.tensor(beta, requires_grad=True)
    rm, rv = ops.tensor(np.zeros(4, np.float32)), ops.tensor(np.ones(4, np.float32))
    y = ops.batch_norm2d(X, G, Be, rm, rv, training=True)
    y.backward(ops.tensor(g))
    bn = torch.nn.BatchNorm2d(4, eps=1e-5, momentum=0.1)
    with torch.no_grad():
        bn.weight.copy_(torch.tensor(gamma))
        bn.bias.copy_(torch.tensor(beta))
    xt = torch.tensor(x, requires_grad=True)
    yt = bn(xt)
    yt.backward(torch.tensor(g))
    np.testing.assert_allclose(ops.to_numpy(y), yt.detach().numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(ops.to_numpy(X.grad), xt.grad.numpy(), rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(ops.to_numpy(G.grad), bn.weight.grad.numpy(), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(ops.to_numpy(Be.grad), bn.bias.grad.numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(ops.to_numpy(rm), bn.running_mean.numpy(), rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(ops.to_numpy(rv), bn.running_var.numpy(), rtol=1e-5, atol=1e-7)
    bn.eval()
    ye = ops.batch_norm2d(ops.tensor(x), G, Be, rm, rv, training=False)
    np.testing.assert_allclose(ops.to_numpy(ye), bn(torch.tensor(x)).detach().numpy(), rtol=1e-5, atol=1e-5)


def test_ops_build_on_a_bound_tensor_type(dev, ops):
    """bind(module) puts the ops' graph on another tensor type with the reference
    Tensor's protocol (here a subclass standing in for nn_engine.Tensor)."""
    from directcompute_torch_b200.tensor import DeviceTensor

    class Other(DeviceTensor):
        __slots__ = ()

    class Mod:
        Tensor = Other
    try:
        assert ops.bind(Mod) is Other
        a = ops.tensor(np.arange(6, dtype=np.float32).reshape(2, 3), requires_grad=True)
        assert type(a) is Other
        y = ops.sum(ops.mul(a, a))
        y.backward()
        assert type(a.grad) is Other or isinstance(a.grad, DeviceTensor)
        np.testing.assert_allclose(ops.to_numpy(a.grad), 2 * np.arange(6, dtype=np.float32).reshape(2, 3))
        with pytest.raises(TypeError):
            ops.bind(object())
    finally:
        ops.bind()
