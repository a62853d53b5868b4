"""RunSequence replayed as a CUDA graph (the reference's ComputeGraph path).

A command list built with ResolveShader (as nn_engine.py:2505-2771 does) is
replayed many times with graphs on (the default: eager once, captured on the
second identical call, launched after that) and off (DCT_SEQ_GRAPH=0); every
replay's outputs must be bit-identical.  A list that names a different buffer,
or runs after the scratch workspace moved, must not replay a stale graph.
"""
import ctypes
import os

import numpy as np
import pytest

from directcompute_torch_b200._abi import SeqCmd
from oracle import shaders as S

pytestmark = pytest.mark.gpu


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


def _c1_sequence(dev, M=256, N=784, seed=60):
    """C1: fwd bias_relu, column sums (bias_grad), full sum; bwd relu_grad, bias_grad."""
    r = np.random.default_rng(seed)
    x = r.standard_normal((M, N)).astype(np.float32)
    b = r.uniform(-0.1, 0.1, N).astype(np.float32)
    h = {"x": dev.buf(x), "b": dev.buf(b), "y": dev.empty(M * N), "col": dev.empty(N), "tot": dev.empty(1),
         "ones": dev.buf(np.ones(M * N, np.float32)), "dx": dev.empty(M * N), "db": dev.empty(N),
         "acc": dev.empty(N)}
    lib = dev.lib
    g = ((M * N + 255) // 256, 1, 1)
    cmds = [
        _cmd(lib, "bias_relu", [h["x"], h["b"]], [h["y"]], g, [M, N]),
        _cmd(lib, "bias_grad", [h["y"]], [h["col"]], (N, 1, 1), [M, N, N, 1]),
        _cmd(lib, "dct_reduce_all", [h["y"]], [h["tot"]], (1, 1, 1), [0, M * N]),
        _cmd(lib, "relu_grad", [h["ones"], h["y"]], [h["dx"]], g, [M * N]),
        _cmd(lib, "bias_grad", [h["dx"]], [h["db"]], (N, 1, 1), [M, N, N, 1]),
        _cmd(lib, "grad_accum", [h["db"]], [h["acc"]], ((N + 255) // 256, 1, 1), [N]),   # changes every replay
    ]
    arr = (SeqCmd * len(cmds))(*cmds)
    return h, arr, x, b


def _replay(dev, arr, n, reps, graph):
    os.environ["DCT_SEQ_GRAPH"] = "1" if graph else "0"
    try:
        for _ in range(reps):
            dev.lib.RunSequence(ctypes.cast(arr, ctypes.c_void_p), n)
        dev.sync()
    finally:
        os.environ.pop("DCT_SEQ_GRAPH", None)


def test_graph_replay_matches_eager(dev):
    dev.clear_error()
    outs = {}
    for graph in (False, True):
        h, arr, x, b = _c1_sequence(dev)
        _replay(dev, arr, len(arr), 7, graph)
        outs[graph] = {k: dev.read(v) for k, v in h.items()}
        assert dev.error()[0] == 0, dev.error()
        dev.free(*h.values())
    for k in outs[False]:
        assert np.array_equal(outs[True][k].view(np.uint32), outs[False][k].view(np.uint32)), k
    # and the replayed values are the oracle's
    M, N = 256, 784
    r = np.random.default_rng(60)
    x = r.standard_normal((M, N)).astype(np.float32)
    b = r.uniform(-0.1, 0.1, N).astype(np.float32)
    y = np.asarray(S.bias_relu(x.ravel(), b, M, N), np.float32)
    assert np.array_equal(outs[True]["y"].view(np.uint32), y.view(np.uint32))
    dx = np.asarray(S.relu_grad(np.ones(M * N, np.float32), y, M * N), np.float32)
    db = dx.reshape(M, N).astype(np.float64).sum(axis=0)
    np.testing.assert_allclose(outs[True]["db"], db, rtol=1e-6)
    np.testing.assert_allclose(outs[True]["acc"], 7 * db, rtol=1e-6)


def test_graph_not_replayed_on_other_buffers_or_moved_workspace(dev):
    dev.clear_error()
    lib = dev.lib
    h, arr, x, b = _c1_sequence(dev)
    _replay(dev, arr, len(arr), 3, True)                    # eager, capture, launch
    y_ref = dev.read(h["y"])
    # the same list, but the input handle now names another buffer (x * 2)
    x2 = dev.buf(2 * x)
    arr[0].srvs[0] = x2
    _replay(dev, arr, len(arr), 1, True)
    y2 = dev.read(h["y"])
    want = np.maximum(2 * x + b[None, :], 0).ravel()
    assert np.array_equal(y2.view(np.uint32), want.astype(np.float32).view(np.uint32))
    assert not np.array_equal(y2, y_ref)
    # grow the scratch workspace with a large reduction, then replay: still correct
    big = dev.empty(1 << 26)
    hb = dev.empty(1 << 16)
    assert lib.dct_reduce(0, big, 1 << 10, 1 << 16, 1, hb, None) == 0
    arr[0].srvs[0] = h["x"]
    _replay(dev, arr, len(arr), 3, True)
    y3 = dev.read(h["y"])
    assert np.array_equal(y3.view(np.uint32), y_ref.view(np.uint32))
    assert dev.error()[0] == 0, dev.error()
    dev.free(x2, big, hb, *h.values())


def test_run_sequence_with_sgd_equals_sequence_then_sgdbatch(dev):
    """RunSequenceWithSGD (engine.cpp:958-977): the command list, then one SGD step over
    the (param, grad) pairs, equals RunSequence followed by SGDBatch bit for bit."""
    dev.clear_error()
    lib = dev.lib
    r = np.random.default_rng(61)
    w0 = r.standard_normal(784).astype(np.float32)
    outs = []
    for fused in (False, True):
        h, arr, x, b = _c1_sequence(dev)
        hw = dev.buf(w0)
        P = (ctypes.c_void_p * 1)(hw)
        G = (ctypes.c_void_p * 1)(h["db"])
        Sz = (ctypes.c_uint * 1)(784)
        os.environ["DCT_SEQ_GRAPH"] = "1"
        try:
            for _ in range(3):
                if fused:
                    lib.RunSequenceWithSGD(ctypes.cast(arr, ctypes.c_void_p), len(arr), P, G, Sz, 1, 0.05, 1.0)
                else:
                    lib.RunSequence(ctypes.cast(arr, ctypes.c_void_p), len(arr))
                    lib.SGDBatch(P, G, Sz, 1, 0.05, 1.0)
            dev.sync()
        finally:
            os.environ.pop("DCT_SEQ_GRAPH", None)
        outs.append((dev.read(hw), dev.read(h["acc"]), dev.read(h["db"])))
        assert dev.error()[0] == 0, dev.error()
        dev.free(hw, *h.values())
    assert np.array_equal(outs[0][0].view(np.uint32), outs[1][0].view(np.uint32))
    assert np.array_equal(outs[0][1].view(np.uint32), outs[1][1].view(np.uint32))
    w = w0.copy()                                                  # db is the same on every replay
    for _ in range(3):
        w = S.sgd(w, outs[1][2], 784, 0.05, 1.0)
    assert np.array_equal(outs[1][0].view(np.uint32), w.view(np.uint32))
    assert not np.array_equal(outs[1][0], w0)
