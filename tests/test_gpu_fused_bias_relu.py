"""The backward of bias + ReLU in one pass (dct_bias_relu_backward, and the
relu_grad -> bias_grad pair fused inside RunSequence) against the two reference
dispatches and the oracle.

BiasReLUFunc.backward (nn_engine.py:1091-1106) dispatches relu_grad
(nn_relu_grad.hlsl:6-9) and then bias_grad (nn_bias_grad.hlsl:8-29) over its
output.  The fused kernel reads grad and the forward output once and writes dx
and the column sums: dx bit-exact against the oracle, db within rel 1e-5 of the
float64 column sums, and both bit-identical to the unfused dispatches.
"""
import ctypes

import numpy as np
import pytest

from directcompute_torch_b200._abi import SeqCmd
from oracle import shaders as S

pytestmark = pytest.mark.gpu

SHAPES = [(256, 784), (1000, 4096), (16384, 4096), (7, 5), (3, 1), (1, 1024), (4097, 12)]


def _inputs(M, N, seed):
    r = np.random.default_rng(seed)
    g = r.standard_normal((M, N)).astype(np.float32)
    y = np.maximum(r.standard_normal((M, N)).astype(np.float32), np.float32(0))
    if y.size > 8:
        y.ravel()[:4] = [np.nan, -0.0, 0.0, 1e-38]          # NaN and signed zeros do not pass the gate
    return g, y


def _unfused(dev, hg, hy, M, N):
    hdx, hdb = dev.empty(M * N), dev.empty(N)
    dev.run("relu_grad", [hg, hy], [hdx], ((M * N + 255) // 256, 1, 1), [M * N])
    dev.run("bias_grad", [hdx], [hdb], (N, 1, 1), [M, N, N, 1])
    return hdx, hdb


@pytest.mark.parametrize("shape", SHAPES)
def test_entry_point_matches_oracle_and_unfused(dev, shape):
    M, N = shape
    g, y = _inputs(M, N, M + N)
    hg, hy = dev.buf(g), dev.buf(y)
    hdx, hdb = dev.empty(M * N), dev.empty(N)
    assert dev.lib.dct_bias_relu_backward(hg, hy, hdx, hdb, M, N) == 0, dev.error()
    dx, db = dev.read(hdx), dev.read(hdb)
    want_dx = S.relu_grad(g.ravel(), y.ravel(), M * N)
    assert np.array_equal(dx.view(np.uint32), want_dx.view(np.uint32))
    want_db = want_dx.astype(np.float64).reshape(M, N).sum(0)
    assert np.all(np.abs(db - want_db) <= 1e-5 * np.abs(want_db) + 1e-30)
    udx, udb = _unfused(dev, hg, hy, M, N)
    assert np.array_equal(dev.read(udx).view(np.uint32), dx.view(np.uint32))
    assert np.array_equal(dev.read(udb).view(np.uint32), db.view(np.uint32))
    dev.free(hg, hy, hdx, hdb, udx, udb)


def test_in_place_and_refusals(dev):
    M, N = 513, 256
    g, y = _inputs(M, N, 3)
    hg, hy, hdb = dev.buf(g), dev.buf(y), dev.empty(N)
    assert dev.lib.dct_bias_relu_backward(hg, hy, hg, hdb, M, N) == 0, dev.error()     # dx = grad, in place
    want_dx = S.relu_grad(g.ravel(), y.ravel(), M * N)
    assert np.array_equal(dev.read(hg).view(np.uint32), want_dx.view(np.uint32))
    assert dev.lib.dct_bias_relu_backward(hg, hy, hg, hg, M, N) == 4               # db aliases dx: ARG
    dev.clear_error()
    assert dev.lib.dct_bias_relu_backward(hg, hy, hg, hdb, M + 1, N) == 3          # too small: SIZE
    dev.clear_error()
    dev.free(hg, hy, hdb)


def _cmd(lib, name, srvs, uavs, groups, words):
    c = SeqCmd()
    c.shader = lib.ResolveShader(name.encode())
    assert c.shader, name
    for i, h in enumerate(srvs):
        c.srvs[i] = h
    for i, h in enumerate(uavs):
        c.uavs[i] = h
    c.srvCount, c.uavCount = len(srvs), len(uavs)
    c.threads[0], c.threads[1], c.threads[2] = groups
    cb = np.array(words, np.uint32).tobytes()
    ctypes.memmove(c.cbData, cb, len(cb))
    c.cbSize = len(cb)
    return c


@pytest.mark.parametrize("shape", [(256, 784), (64, 10), (300, 4099)])
def test_run_sequence_fuses_the_pair(dev, shape):
    """A command list with relu_grad then bias_grad over its dx (the backward that
    BiasReLUFunc records) replays, eager and as a graph, to the unfused results."""
    M, N = shape
    g, y = _inputs(M, N, 11)
    hg, hy, hdx, hdb = dev.buf(g), dev.buf(y), dev.empty(M * N), dev.empty(N)
    lib = dev.lib
    cmds = [_cmd(lib, "relu_grad", [hg, hy], [hdx], ((M * N + 255) // 256, 1, 1), [M * N]),
            _cmd(lib, "bias_grad", [hdx], [hdb], (N, 1, 1), [M, N, N, 1])]
    arr = (SeqCmd * 2)(*cmds)
    udx, udb = _unfused(dev, hg, hy, M, N)
    want_dx, want_db = dev.read(udx), dev.read(udb)
    for _ in range(4):                                  # eager, capture, then graph launches
        lib.RunSequence(ctypes.cast(arr, ctypes.c_void_p), 2)
        dev.sync()
        assert dev.error()[0] == 0, dev.error()
        assert np.array_equal(dev.read(hdx).view(np.uint32), want_dx.view(np.uint32))
        assert np.array_equal(dev.read(hdb).view(np.uint32), want_db.view(np.uint32))
        lib.ClearBuffer(hdx)
        lib.ClearBuffer(hdb)
    dev.free(hg, hy, hdx, hdb, udx, udb)


def _bias_inputs(M, N, seed):
    r = np.random.default_rng(seed)
    x = r.standard_normal((M, N)).astype(np.float32)
    b = r.uniform(-0.1, 0.1, N).astype(np.float32)
    if x.size > 8:
        x.ravel()[:3] = [np.nan, -b[1], -0.0]                # NaN -> 0, an exact zero sum, -0 + b
    return x, b


@pytest.mark.parametrize("shape", [(256, 784), (64, 10), (300, 4099), (1, 5), (4097, 12)])
def test_run_sequence_fuses_bias_relu_with_its_column_sums(dev, shape):
    """bias_relu then bias_grad over its output (the C1 forward) runs as one pass
    inside RunSequence: y and the column sums bit-identical to the two dispatches,
    y bit-exact against the oracle, eager and as a graph."""
    M, N = shape
    x, b = _bias_inputs(M, N, 21)
    hx, hb, hy, hc = dev.buf(x), dev.buf(b), dev.empty(M * N), dev.empty(N)
    lib = dev.lib
    g = ((M * N + 255) // 256, 1, 1)
    arr = (SeqCmd * 2)(_cmd(lib, "bias_relu", [hx, hb], [hy], g, [M, N]),
                       _cmd(lib, "bias_grad", [hy], [hc], (N, 1, 1), [M, N, N, 1]))
    uy, uc = dev.empty(M * N), dev.empty(N)
    dev.run("bias_relu", [hx, hb], [uy], g, [M, N])
    dev.run("bias_grad", [uy], [uc], (N, 1, 1), [M, N, N, 1])
    want_y, want_c = dev.read(uy), dev.read(uc)
    assert np.array_equal(want_y.view(np.uint32), S.bias_relu(x.ravel(), b, M, N).view(np.uint32))
    for _ in range(4):                                  # eager, capture, then graph launches
        lib.RunSequence(ctypes.cast(arr, ctypes.c_void_p), 2)
        dev.sync()
        assert dev.error()[0] == 0, dev.error()
        assert np.array_equal(dev.read(hy).view(np.uint32), want_y.view(np.uint32))
        assert np.array_equal(dev.read(hc).view(np.uint32), want_c.view(np.uint32))
        lib.ClearBuffer(hy)
        lib.ClearBuffer(hc)
    dev.free(hx, hb, hy, hc, uy, uc)


@pytest.mark.parametrize("shape", [(256, 784), (300, 4099)])
def test_run_sequence_fuses_the_backward_with_grad_accum(dev, shape):
    """relu_grad, bias_grad and grad_accum over those column sums (the C1 backward)
    run as one pass plus its fold: dx, db and the accumulator bit-identical to the
    three dispatches after every replay."""
    M, N = shape
    g, y = _inputs(M, N, 31)
    hg, hy, hdx, hdb, hacc = dev.buf(g), dev.buf(y), dev.empty(M * N), dev.empty(N), dev.empty(N)
    lib = dev.lib
    gr = ((M * N + 255) // 256, 1, 1)
    arr = (SeqCmd * 3)(_cmd(lib, "relu_grad", [hg, hy], [hdx], gr, [M * N]),
                       _cmd(lib, "bias_grad", [hdx], [hdb], (N, 1, 1), [M, N, N, 1]),
                       _cmd(lib, "grad_accum", [hdb], [hacc], ((N + 255) // 256, 1, 1), [N]))
    udx, udb, uacc = dev.empty(M * N), dev.empty(N), dev.empty(N)
    for rep in range(4):                                # eager, capture, then graph launches
        dev.run("relu_grad", [hg, hy], [udx], gr, [M * N])
        dev.run("bias_grad", [udx], [udb], (N, 1, 1), [M, N, N, 1])
        dev.run("grad_accum", [udb], [uacc], ((N + 255) // 256, 1, 1), [N])
        lib.RunSequence(ctypes.cast(arr, ctypes.c_void_p), 3)
        dev.sync()
        assert dev.error()[0] == 0, dev.error()
        for h, u in ((hdx, udx), (hdb, udb), (hacc, uacc)):
            assert np.array_equal(dev.read(h).view(np.uint32), dev.read(u).view(np.uint32)), rep
    dev.free(hg, hy, hdx, hdb, hacc, udx, udb, uacc)
