"""Reference elementwise shaders through RunShader vs the NumPy oracle: BIT-EXACT.

Each case packs the cbuffer words exactly as nn_engine.py does and dispatches
the reference's group counts; sizes cover n = 1, odd tails, non-multiples of 4
and special values (+-0, +-inf, NaN, subnormals).
"""
import numpy as np
import pytest

from oracle import shaders as S
from tests.devhelp import f2u

pytestmark = pytest.mark.gpu

SIZES = [1, 3, 255, 257, 4097, 100003]


def _x(n, seed, special=True):
    r = np.random.default_rng(seed)
    x = (r.standard_normal(n) * 3).astype(np.float32)
    if special and n >= 16:
        x[:8] = [0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 6.0]
    return x


def _same(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    assert a.shape == b.shape
    both_nan = np.isnan(a) & np.isnan(b)
    eq = (a.view(np.uint32) == b.view(np.uint32)) | both_nan
    if not eq.all():
        i = np.flatnonzero(~eq)[:5]
        raise AssertionError(f"{(~eq).sum()} mismatches, e.g. idx {i}: got {a[i]} want {b[i]}")


def _g(n, per=256):
    return ((n + per - 1) // per, 1, 1)


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("relu", [False, True])
def test_add_bias(dev, n, relu):
    N = max(1, min(n, 784))
    M = max(1, n // N)
    A = _x(M * N, 1)
    B = _x(N, 2, special=False)
    ha, hb, hc = dev.buf(A), dev.buf(B), dev.empty(M * N)
    name = "bias_relu" if relu else "add_bias"
    dev.run(name, [ha, hb], [hc], _g(M * N), [M, N])
    want = (S.bias_relu if relu else S.add_bias)(A, B, M, N)
    _same(dev.read(hc), want)
    dev.free(ha, hb, hc)


@pytest.mark.parametrize("n", SIZES)
def test_relu_no_cbuffer(dev, n):
    x = _x(n, 3)
    hx, hy = dev.buf(x), dev.empty(n)
    dev.run("relu", [hx], [hy], _g(n))
    _same(dev.read(hy), S.relu(x, n))
    dev.free(hx, hy)


def test_relu_reads_past_input_as_zero(dev):
    x = _x(100, 4)
    hx, hy = dev.buf(x), dev.empty(300, fill=7.0)
    dev.run("relu", [hx], [hy], _g(300))
    _same(dev.read(hy), S.relu(x, 300))
    dev.free(hx, hy)


UNARY_REF = {
    "relu6": lambda x, n, a: S.relu6(x, n),
    "leaky_relu": lambda x, n, a: S.leaky_relu(x, n, a),
}
BINARY_REF = {
    "relu_grad": lambda g, x, n, a: S.relu_grad(g, x, n),
    "relu6_grad": lambda g, x, n, a: S.relu6_grad(g, x, n),
    "leaky_relu_grad": lambda g, x, n, a: S.leaky_relu_grad(g, x, n, a),
    "sigmoid_grad": lambda g, y, n, a: S.sigmoid_grad(g, y, n),
}


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("name", sorted(UNARY_REF))
def test_unary_shaders(dev, name, n):
    x = _x(n, 5)
    alpha = np.float32(0.1)
    hx, hy = dev.buf(x), dev.empty(n)
    dev.run(name, [hx], [hy], _g(n), [n, f2u(alpha)])
    _same(dev.read(hy), UNARY_REF[name](x, n, alpha))
    dev.free(hx, hy)


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("name", sorted(BINARY_REF))
def test_grad_shaders(dev, name, n):
    g, x = _x(n, 6), _x(n, 7)
    if name == "sigmoid_grad":
        x = (1 / (1 + np.exp(-x.astype(np.float64)))).astype(np.float32)
    alpha = np.float32(0.2)
    hg, hx, hy = dev.buf(g), dev.buf(x), dev.empty(n)
    dev.run(name, [hg, hx], [hy], _g(n), [n, f2u(alpha)])
    _same(dev.read(hy), BINARY_REF[name](g, x, n, alpha))
    dev.free(hg, hx, hy)


@pytest.mark.parametrize("n", SIZES)
def test_add_scale_add_grad_accum(dev, n):
    a, b = _x(n, 8), _x(n, 9)
    ha, hb, hc = dev.buf(a), dev.buf(b), dev.empty(n)
    dev.run("add", [ha, hb], [hc], _g(n), [n, 1])
    _same(dev.read(hc), S.add(a, b, n, 1))
    al, be = np.float32(0.95), np.float32(-0.5)
    dev.run("scale_add", [ha, hb], [hc], _g(n), [n, f2u(al), f2u(be)])
    _same(dev.read(hc), S.scale_add(a, b, n, al, be))
    # in place, as Muon does: m = momentum*m + g (t0 and u0 are the same buffer)
    dev.run("scale_add", [hc, hb], [hc], _g(n), [n, f2u(al), f2u(np.float32(1.0))])
    _same(dev.read(hc), S.scale_add(S.scale_add(a, b, n, al, be), b, n, al, 1.0))
    acc = dev.read(hc).copy()
    dev.run("grad_accum", [ha], [hc], _g(n), [n])
    _same(dev.read(hc), S.grad_accum(acc, a, n))
    dev.free(ha, hb, hc)


@pytest.mark.parametrize("n", SIZES)
def test_sigmoid_within_2ulp(dev, n):
    from oracle.newops import ulp_diff
    x = _x(n, 10)
    hx, hy = dev.buf(x), dev.empty(n)
    dev.run("sigmoid", [hx], [hy], _g(n), [n])
    got = dev.read(hy)
    want = S.sigmoid_f64(x, n)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert ulp_diff(got[~nan], want[~nan]).max() <= 2
    dev.free(hx, hy)


@pytest.mark.parametrize("shape", [(2, 3, 4), (8, 16, 49), (4, 64, 3136)])
def test_global_avg_pool_backward(dev, shape):
    n, c, s = shape
    g = _x(n * c, 11, special=False)
    hg, hy = dev.buf(g), dev.empty(n * c * s)
    dev.run("global_avg_pool_backward", [hg], [hy], _g(n * c * s), [n, c, s])
    _same(dev.read(hy), S.global_avg_pool_backward(g, n, c, s))
    dev.free(hg, hy)


def test_accumulate_scalar(dev):
    hs, hd = dev.buf(np.float32([1.25])), dev.buf(np.float32([2.5]))
    dev.run("accumulate_scalar", [hs], [hd], (1, 1, 1))
    dev.run("accumulate_scalar", [hs], [hd], (1, 1, 1))
    assert dev.read(hd)[0] == np.float32(5.0)
    dev.free(hs, hd)


@pytest.mark.parametrize("BK", [(4, 10), (33, 17), (256, 1000)])
def test_softmax_ce_grad_exact(dev, BK):
    B, K = BK
    r = np.random.default_rng(12)
    p = r.random((B, K), dtype=np.float32)
    lab = r.integers(0, K, B).astype(np.float32)
    hp, hl, hg = dev.buf(p), dev.buf(lab), dev.empty(B * K)
    dev.run("softmax_ce_grad", [hp, hl], [hg], ((K + 15) // 16, (B + 15) // 16, 1), [B, K])
    _same(dev.read(hg).reshape(B, K), S.softmax_ce_grad(p.ravel(), lab, B, K))
    dev.free(hp, hl, hg)


# (3, 777): the scalar kernel; (4, 4096) and (5, 1000): the float4 chunked kernel
@pytest.mark.parametrize("b,size", [(3, 777), (4, 4096), (5, 1000)])
def test_dice_grad_exact_given_sums(dev, b, size):
    r = np.random.default_rng(13)
    p = r.random(b * size, dtype=np.float32)
    t = (r.random(b * size) > 0.5).astype(np.float32)
    sums = S.dice_sums(p, t, b, size).astype(np.float32).ravel()
    hp, ht, hs, hd = dev.buf(p), dev.buf(t), dev.buf(sums), dev.empty(b * size)
    dev.run("dice_loss_grad", [hp, ht, hs], [hd], _g(b * size), [b, size])
    _same(dev.read(hd), S.dice_loss_grad(p, t, sums, b, size))
    dev.free(hp, ht, hs, hd)


def test_unknown_shader_is_silent_noop(dev):
    dev.clear_error()
    h = dev.empty(4, fill=3.0)
    dev.run("matmul_universal", [h], [h], (1, 1, 1), [1, 1, 1, 0])
    assert (dev.read(h) == 3.0).all()
    code, msg = dev.error()
    assert code == 6 and "matmul_universal" in msg
    dev.free(h)


def test_undersized_buffer_rejected_not_overrun(dev):
    dev.clear_error()
    a, b, c = dev.empty(10, 1.0), dev.empty(10, 2.0), dev.empty(5, 9.0)
    dev.run("add", [a, b], [c], (1, 1, 1), [10, 1])
    code, msg = dev.error()
    assert code == 3, msg
    assert (dev.read(c) == 9.0).all()
    dev.free(a, b, c)
