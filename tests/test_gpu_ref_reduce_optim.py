"""Reference reduction / softmax / optimizer / BatchNorm shaders through RunShader.

Sums are held to rel 1e-5 of the float64-accumulated oracle (they come out
~1e-7); elementwise stages fed by given statistics are bit-exact; counts and
indices are exact.
"""
import ctypes

import numpy as np
import pytest

from oracle import shaders as S
from tests.devhelp import f2u

pytestmark = pytest.mark.gpu


def _same(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    eq = (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
    assert eq.all(), f"{(~eq).sum()} mismatches: got {a[~eq][:4]} want {b[~eq][:4]}"


def _close(got, want, rtol=1e-5, atol=0.0):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    assert (err <= rtol * np.abs(want) + atol).all(), f"max err {err.max()} (rel {(err / np.maximum(np.abs(want), 1e-30)).max()})"


@pytest.mark.parametrize("MN", [(1, 1), (256, 784), (33, 17), (16384, 4096)])
def test_bias_grad_colsum(dev, MN):
    M, N = MN
    r = np.random.default_rng(M + N)
    g = r.standard_normal((M, N)).astype(np.float32)
    hg, ho = dev.buf(g), dev.empty(N)
    dev.run("bias_grad", [hg], [ho], (N, 1, 1), [M, N, N, 1])
    _close(dev.read(ho), g.astype(np.float64).sum(0), atol=1e-6 * np.sqrt(M))
    dev.free(hg, ho)


@pytest.mark.parametrize("cfg", [(100, 6, 1, 100), (10, 7, 3, 31)])
def test_bias_grad_strided(dev, cfg):
    # conv backward uses stride_i=1, stride_id=totalCol (engine.cpp:844-855)
    batch, classes, si, sc = cfg
    r = np.random.default_rng(3)
    n = (batch - 1) * si + (classes - 1) * sc + 1
    g = r.standard_normal(n).astype(np.float32)
    hg, ho = dev.buf(g), dev.empty(classes)
    dev.run("bias_grad", [hg], [ho], (classes, 1, 1), [batch, classes, si, sc])
    _close(dev.read(ho), S.bias_grad(g, batch, classes, si, sc).astype(np.float64), rtol=1e-6, atol=1e-6)
    dev.free(hg, ho)


@pytest.mark.parametrize("shape", [(2, 3, 16), (4, 32, 49), (8, 64, 3136)])
def test_global_avg_pool(dev, shape):
    n, c, s = shape
    x = np.random.default_rng(1).standard_normal(n * c * s).astype(np.float32)
    hx, ho = dev.buf(x), dev.empty(n * c)
    dev.run("global_avg_pool", [hx], [ho], (n * c, 1, 1), [n, c, s])
    _close(dev.read(ho), x.astype(np.float64).reshape(n * c, s).mean(1), atol=1e-7)
    dev.free(hx, ho)


def test_rms_and_clip_reduction(dev):
    r = np.random.default_rng(2)
    a = r.standard_normal(300001).astype(np.float32)
    ha, ho = dev.buf(a), dev.empty(1)
    dev.run("rms", [ha], [ho], (1, 1, 1), [a.size])
    _close(dev.read(ho), [np.sqrt((a.astype(np.float64) ** 2).mean())], rtol=1e-6)
    k = (a.size + 255) // 256
    hp = dev.empty(k + 5)
    dev.run("grad_sq_reduce", [ha], [hp], (k, 1, 1), [a.size, 5])
    part = dev.read(hp)
    _close(part[5:], S.grad_sq_reduce(a, a.size, k).astype(np.float64), rtol=1e-6)
    hns = dev.empty(2)
    dev.run("grad_norm_final", [hp], [hns], (1, 1, 1), [k + 5, f2u(1.0)])
    norm, scale = dev.read(hns)
    want_norm = np.sqrt((part.astype(np.float64)).sum())
    _close([norm], [want_norm], rtol=1e-6)
    assert scale == S.grad_norm_final(part, k + 5, 1.0)[1]
    dev.free(ha, ho, hp, hns)


@pytest.mark.parametrize("BK", [(4, 10), (100, 1000), (17, 3000)])
def test_softmax_and_loss_names(dev, BK):
    from oracle.newops import ulp_diff
    B, K = BK
    r = np.random.default_rng(B)
    x = (3 * r.standard_normal((B, K))).astype(np.float32)
    lab = r.integers(0, K, B).astype(np.float32)
    hx, hl, hp, hloss = dev.buf(x), dev.buf(lab), dev.empty(B * K), dev.empty(1)
    dev.run("softmax", [hx], [hp], ((B + 15) // 16, 1, 1), [B, K])
    assert ulp_diff(dev.read(hp), S.softmax_f64(x.ravel(), B, K).ravel()).max() <= 4
    dev.run("loss", [hx, hl], [hloss], (1, 1, 1), [B, K])
    _close(dev.read(hloss), [S.ce_loss_f64(x.ravel(), lab, B, K)], rtol=1e-6)
    dev.free(hx, hl, hp, hloss)


def test_argmax_correct_counts(dev):
    r = np.random.default_rng(5)
    B, K = 1000, 10
    x = r.standard_normal((B, K)).astype(np.float32)
    x[0, :] = 1.0                       # ties -> index 0
    x[1, 0] = np.nan                    # NaN at column 0 -> index 0
    x[2, 3] = np.nan                    # other NaNs are never chosen
    lab = x.argmax(1).astype(np.float32)
    lab[::3] = (lab[::3] + 1) % K
    lab[1] = 0
    hx, hl = dev.buf(x), dev.buf(lab)
    hc = dev.buf(np.zeros(1, np.uint32))
    for _ in range(2):
        dev.run("argmax_correct", [hx, hl], [hc], ((B + 255) // 256, 1, 1), [B, K])
    want = S.argmax_correct(x.ravel(), lab, B, K)
    assert int(dev.read(hc, np.uint32)[0]) == 2 * want
    dev.free(hx, hl, hc)


def test_sgd_shaders_bitexact(dev):
    r = np.random.default_rng(6)
    n = 100001
    w = r.standard_normal(n).astype(np.float32)
    g = (r.standard_normal(n) * 2).astype(np.float32)
    hw, hg = dev.buf(w), dev.buf(g)
    dev.run("sgd", [hg], [hw], ((n + 255) // 256, 1, 1), [n, f2u(0.01), f2u(1.0)])
    w = S.sgd(w, g, n, 0.01, 1.0)
    _same(dev.read(hw), w)
    ns = np.float32([3.0, 0.25])
    hns = dev.buf(ns)
    dev.run("sgd_clipped", [hg, hns], [hw], ((n + 255) // 256, 1, 1), [n, f2u(0.05)])
    _same(dev.read(hw), S.sgd_clipped(w, g, n, 0.05, ns[1]))
    dev.free(hw, hg, hns)


def test_adam_shader_bitexact(dev):
    r = np.random.default_rng(7)
    n = 77777
    w = r.standard_normal(n).astype(np.float32)
    g = r.standard_normal(n).astype(np.float32)
    m = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    hw, hm, hv, hg = dev.buf(w), dev.buf(m), dev.buf(v), dev.buf(g)
    for t in (1, 2):
        step = S.adam_step_size(0.01, 0.9, 0.999, t)
        words = [n, f2u(step), f2u(0.9), f2u(0.999), f2u(1e-8), f2u(0.01 * 0.01), f2u(1.0)]
        dev.run("adam", [hg], [hw, hm, hv], ((n + 255) // 256, 1, 1), words)
        w, m, v = S.adam(w, m, v, g, n, step, 0.9, 0.999, 1e-8, np.float32(0.01 * 0.01), 1.0)
    _same(dev.read(hw), w)
    _same(dev.read(hm), m)
    _same(dev.read(hv), v)
    dev.free(hw, hm, hv, hg)


def _arr(vals, t=ctypes.c_void_p):
    return (t * len(vals))(*vals)


def test_sgd_batch_and_clipped(dev):
    r = np.random.default_rng(8)
    sizes = [10, 1000, 4097, 70000, 3]
    ws = [r.standard_normal(s).astype(np.float32) for s in sizes]
    gs = [(r.standard_normal(s) * 3).astype(np.float32) for s in sizes]
    hw = [dev.buf(w) for w in ws]
    hg = [dev.buf(g) for g in gs]
    lib = dev.lib
    lib.SGDBatch(_arr(hw), _arr(hg), _arr(sizes, ctypes.c_uint), len(sizes), 0.1, 1.0)
    for i, s in enumerate(sizes):
        ws[i] = S.sgd(ws[i], gs[i], s, 0.1, 1.0)
        _same(dev.read(hw[i]), ws[i])
    norm = lib.SGDBatchClipped(_arr(hw), _arr(hg), _arr(sizes, ctypes.c_uint), len(sizes), 0.1, 5.0)
    want = np.sqrt(sum((g.astype(np.float64) ** 2).sum() for g in gs))
    _close([norm], [want], rtol=1e-6)
    scale = np.float32(np.float64(np.float32(5.0)) / (np.float64(np.float32(norm)) + np.float64(np.float32(1e-6))))
    for i, s in enumerate(sizes):
        _same(dev.read(hw[i]), S.sgd_clipped(ws[i], gs[i], s, 0.1, scale))
    dev.free(*hw, *hg)


@pytest.mark.parametrize("shape", [(2, 3, 4, 4), (4, 16, 7, 7), (8, 32, 56, 56)])
def test_batchnorm_reference_shaders(dev, shape):
    N, C, H, W = shape
    Sx = H * W
    r = np.random.default_rng(9)
    x = (0.5 + 2 * r.standard_normal(shape)).astype(np.float32).ravel()
    dy = r.standard_normal(shape).astype(np.float32).ravel()
    gamma = r.random(C, dtype=np.float32)
    beta = r.random(C, dtype=np.float32)
    rm0, rv0 = np.zeros(C, np.float32), np.ones(C, np.float32)
    hx, hdy, hgm, hbt = dev.buf(x), dev.buf(dy), dev.buf(gamma), dev.buf(beta)
    hmean, hvar, hrm, hrv = dev.empty(C), dev.empty(C), dev.buf(rm0), dev.buf(rv0)
    dev.run("batchnorm_mean_var", [hx], [hmean, hvar, hrm, hrv], (C, 1, 1), [N, C, Sx, 1, f2u(0.1)])
    mean64, var64 = S.batchnorm_mean_var(x, N, C, Sx)
    mean, var = dev.read(hmean), dev.read(hvar)
    _close(mean, mean64, rtol=1e-6, atol=1e-7)
    _close(var, var64, rtol=1e-6)
    rm, rv = S.batchnorm_running(rm0, rv0, mean64, var64, N, Sx, 0.1)
    _close(dev.read(hrm), rm, rtol=1e-6, atol=1e-8)
    _close(dev.read(hrv), rv, rtol=1e-6)
    hy = dev.empty(x.size)
    eps = np.float32(1e-5)
    dev.run("batchnorm_forward", [hx, hmean, hvar, hgm, hbt], [hy], ((x.size + 255) // 256, 1, 1),
            [N, C, Sx, f2u(eps)])
    _same(dev.read(hy), S.batchnorm_forward(x, mean, var, gamma, beta, N, C, Sx, eps))
    hdg, hdb = dev.empty(C), dev.empty(C)
    dev.run("batchnorm_backward_reduce", [hx, hdy, hmean, hvar], [hdg, hdb], (C, 1, 1), [N, C, Sx, f2u(eps)])
    dg, db = S.batchnorm_backward_reduce(x, dy, mean, var, N, C, Sx, eps)
    gdg, gdb = dev.read(hdg), dev.read(hdb)
    _close(gdg, dg, rtol=1e-5, atol=1e-6 * np.sqrt(N * Sx))
    _close(gdb, db, rtol=1e-5, atol=1e-6 * np.sqrt(N * Sx))
    hdx = dev.empty(x.size)
    dev.run("batchnorm_backward_dx", [hx, hdy, hmean, hvar, hgm, hdg, hdb], [hdx], ((x.size + 255) // 256, 1, 1),
            [N, C, Sx, f2u(eps)])
    _same(dev.read(hdx), S.batchnorm_backward_dx(x, dy, mean, var, gamma, gdg, gdb, N, C, Sx, eps))
    dev.free(hx, hdy, hgm, hbt, hmean, hvar, hrm, hrv, hy, hdg, hdb, hdx)


# (4, 12288): float4 chunks + the chunk fold; (3, 777): scalar, one chunk a
# sample; (2, 50001): scalar chunks + fold; (700, 4096): one float4 chunk a sample
@pytest.mark.parametrize("b,size", [(4, 3 * 64 * 64), (3, 777), (2, 50001), (700, 4096)])
def test_dice_loss_and_sums(dev, b, size):
    r = np.random.default_rng(10)
    p = r.random(b * size, dtype=np.float32)
    t = (r.random(b * size) > 0.5).astype(np.float32)
    hp, ht, ho, hs = dev.buf(p), dev.buf(t), dev.empty(b), dev.empty(3 * b)
    dev.run("dice_loss", [hp, ht], [ho], (b, 1, 1), [b, size])
    _close(dev.read(ho), S.dice_loss(p, t, b, size), rtol=1e-6)
    dev.run("dice_loss_sums", [hp, ht], [hs], (b, 1, 1), [b, size])
    _close(dev.read(hs), S.dice_sums(p, t, b, size).ravel(), rtol=1e-6)
    dev.free(hp, ht, ho, hs)
