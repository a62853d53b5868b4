"""Layout ops beside the path, through libdct_cuda.so's C-ABI, against the oracle.

Upsample (nn_upsample*.hlsl), channel concat / slice (nn_concat_insert.hlsl,
nn_slice.hlsl), max pooling (nn_maxpool_*.hlsl and MaxPoolForwardFused /
MaxPoolBackwardFused, engine.cpp:880-929) and the conv reshapes
(nn_conv_reshape.hlsl, nn_conv_grad_reshape*.hlsl), dispatched by shader name
with the reference's cbuffer words and group counts.  Every result is
bit-exact except tanh (<= 2 ulp of the float64 value); a NaN matches any NaN
and pooling indices are compared bit for bit.  Each op runs on shapes
that take its 128-bit path and on ragged shapes and partial group counts that
take the scalar path.
"""
import ctypes

import numpy as np
import pytest

from oracle import shaders as S
from oracle.newops import ulp_diff

pytestmark = pytest.mark.gpu

U32 = np.uint32


def _bits(a):
    return np.asarray(a, np.float32).view(U32)


def _same(got, want):
    """Bit-exact, except that a NaN matches any NaN (payloads are not part of the result)."""
    assert got.shape == want.shape
    bad = np.flatnonzero((_bits(got) != _bits(want)) & ~(np.isnan(got) & np.isnan(want)))
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}: {got[bad[:3]]} vs {want[bad[:3]]}"


@pytest.fixture(autouse=True)
def _clean(dev):
    dev.clear_error()
    yield
    code, msg = dev.error()
    assert code == 0, msg


# ---- upsample ---------------------------------------------------------------------
@pytest.mark.parametrize("B,C,H,W,sH,sW,full", [
    (2, 3, 16, 8, 2, 2, True),       # input-major float4 path (inW % 4 == 0, exact scales)
    (2, 2, 4, 8, 3, 1, True),        # input-major, scale 1 across
    (1, 2, 4, 4, 1, 4, True),        # input-major, scale 4 across
    (2, 3, 5, 4, 2, 3, True),        # output-major float4 path (outW % 4 == 0)
    (3, 2, 5, 7, 3, 2, True),        # outW = 14: scalar path
    (2, 3, 6, 9, 1, 4, True),
    (2, 3, 16, 8, 2, 2, False),      # partial group count: scalar path
])
def test_upsample_forward(dev, B, C, H, W, sH, sW, full):
    rng = np.random.default_rng(B * 100 + H)
    x = rng.standard_normal(B * C * H * W).astype(np.float32)
    oH, oW = H * sH, W * sW
    total = B * C * oH * oW
    groups = (total + 255) // 256 if full else max(1, total // 256 - 2)
    hx, hy = dev.buf(x), dev.empty(total, fill=-7.0)
    dev.run("upsample", [hx], [hy], (groups, 1, 1), [B, C, H, W, oH, oW, sH, sW])
    got = dev.read(hy)
    want = np.full(total, -7.0, np.float32)
    r = S.upsample(x, B, C, H, W, oH, oW, sH, sW, limit=groups * 256)
    want[: r.size] = r
    _same(got, want)
    dev.free(hx, hy)


@pytest.mark.parametrize("B,C,H,W,sH,sW,oH,oW,full", [
    (2, 3, 8, 16, 2, 2, 16, 32, True),    # 2x2 float4 path
    (2, 3, 8, 6, 2, 2, 16, 12, True),     # inW % 4 != 0: scalar path
    (3, 2, 5, 7, 3, 2, 15, 14, True),
    (1, 2, 3, 4, 2, 2, 5, 7, True),       # output smaller than in*scale: block tails skipped
    (2, 3, 8, 16, 2, 2, 16, 32, False),
])
def test_upsample_backward(dev, B, C, H, W, sH, sW, oH, oW, full):
    rng = np.random.default_rng(oH * 7 + W)
    dy = rng.standard_normal(B * C * oH * oW).astype(np.float32)
    dy[::13] = -0.0                                            # signed zeros keep the shader's 0.0f start
    total = B * C * H * W
    groups = (total + 255) // 256 if full else max(1, total // 256 - 1)
    hdy, hdx = dev.buf(dy), dev.empty(total, fill=5.0)
    dev.run("upsample_backward", [hdy], [hdx], (groups, 1, 1), [B, C, H, W, oH, oW, sH, sW])
    want = np.full(total, 5.0, np.float32)
    r = S.upsample_backward(dy, B, C, H, W, oH, oW, sH, sW, limit=groups * 256)
    want[: r.size] = r
    _same(dev.read(hdx), want)
    dev.free(hdy, hdx)


# ---- concat / slice -------------------------------------------------------------------
@pytest.mark.parametrize("B,cins,S_,full", [
    (2, (3, 5), 64, True),            # every row a multiple of 4: 128-bit path
    (3, (2, 1, 4), 15, True),         # ragged rows: scalar path
    (2, (3, 5), 64, False),
])
def test_concat_then_slice(dev, B, cins, S_, full):
    rng = np.random.default_rng(sum(cins) + S_)
    cout = sum(cins)
    parts = [rng.standard_normal(B * c * S_).astype(np.float32) for c in cins]
    hout = dev.empty(B * cout * S_, fill=np.nan)
    want = np.full(B * cout * S_, np.nan, np.float32)
    off = 0
    hs = []
    for c, a in zip(cins, parts):
        n = B * c * S_
        groups = (n + 255) // 256 if full else max(1, (n + 255) // 256 - 1)
        h = dev.buf(a)
        hs.append(h)
        dev.run("concat_insert", [h], [hout], (groups, 1, 1), [B, c, S_, cout, off])
        S.concat_insert(want, a, B, c, S_, cout, off, limit=groups * 256)
        off += c
    _same(dev.read(hout), want)
    off = 0
    for c in cins:
        n = B * c * S_
        groups = (n + 255) // 256 if full else max(1, (n + 255) // 256 - 1)
        hd = dev.empty(n, fill=3.0)
        dev.run("slice", [hout], [hd], (groups, 1, 1), [B, c, S_, cout, off])
        w = np.full(n, 3.0, np.float32)
        r = S.slice_channels(want, B, c, S_, cout, off, limit=groups * 256)
        w[: r.size] = r
        _same(dev.read(hd), w)
        dev.free(hd)
        off += c
    dev.free(hout, *hs)


# ---- max pooling ----------------------------------------------------------------------
def _pool_input(rng, B, C, H, W):
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    x[0, 0, :3, :3] = -np.inf                   # never beats -1e30: index 0xFFFFFFFF
    x[0, min(1, C - 1), 2:5, 2:5] = np.nan      # never selected
    x[-1, -1, :2, :] = np.float32(-2e30)
    x[-1, 0, 4, 4:6] = 3.5                      # a tie: the first one wins
    return x.ravel()


@pytest.mark.parametrize("B,C,H,W,p,s,gsub", [
    (2, 3, 16, 32, 2, 2, 0),      # 2x2 float4 path
    (2, 3, 9, 11, 2, 2, 0),       # ragged: scalar path
    (2, 3, 10, 9, 3, 3, 0),
    (2, 3, 9, 11, 3, 2, 0),       # overlapping windows
    (2, 3, 8, 10, 2, 3, 0),       # gaps between windows
    (2, 3, 40, 40, 2, 2, 1),      # partial group counts
])
def test_maxpool_forward_shader(dev, B, C, H, W, p, s, gsub):
    rng = np.random.default_rng(H * W + p)
    x = _pool_input(rng, B, C, H, W)
    oH, oW = (H - p) // s + 1, (W - p) // s + 1
    n = B * C * oH * oW
    g = ((oW + 15) // 16, (oH + 15) // 16, B * C - gsub)
    hx, ho, hi = dev.buf(x), dev.empty(n, fill=1.25), dev.empty(n, fill=1.5)
    dev.run("maxpool_forward", [hx], [ho, hi], g, [B, C, H, W, p, s, oH, oW])
    want_v = np.full(n, 1.25, np.float32)
    want_i = np.full(n, 1.5, np.float32).view(U32).copy()
    o, v, idx = S.maxpool_forward(x, B, C, H, W, p, s, oH, oW, lim_w=g[0] * 16, lim_h=g[1] * 16, lim_bc=g[2])
    want_v[o] = v
    want_i[o] = idx
    _same(dev.read(ho), want_v)
    assert np.array_equal(dev.read(hi, U32), want_i)
    if gsub == 0 and (H, W, p) == (16, 32, 2):
        assert (want_i == 0xFFFFFFFF).any()
    dev.free(hx, ho, hi)


def test_maxpool_backward_shader_scatter(dev):
    rng = np.random.default_rng(5)
    B, C, oH, oW, nin = 2, 3, 5, 6, 2 * 3 * 10 * 12
    n = B * C * oH * oW
    dz = rng.standard_normal(n).astype(np.float32)
    idx = rng.permutation(nin)[:n].astype(U32)          # distinct targets
    idx[::7] = 0xFFFFFFFF                               # no index: no write
    idx[3] = nin + 100                                  # past the buffer: dropped
    hdz, hidx, hd = dev.buf(dz), dev.buf(idx), dev.empty(nin, fill=9.0)
    dev.run("maxpool_backward", [hdz, hidx], [hd], ((oW + 15) // 16, (oH + 15) // 16, B * C), [B, C, oH, oW])
    want = S.maxpool_backward(np.full(nin, 9.0, np.float32), dz, idx, B, C, oH, oW)
    _same(dev.read(hd), want)
    dev.free(hdz, hidx, hd)


def _fused_forward(dev, hx, B, C, H, W, p, s):
    pidx = ctypes.c_void_p()
    out = dev.lib.MaxPoolForwardFused(hx, B, C, H, W, p, s, ctypes.byref(pidx))
    assert out and pidx.value, dev.error()
    return out, pidx.value


@pytest.mark.parametrize("B,C,H,W,p,s", [
    (2, 3, 16, 32, 2, 2),         # one-pass 2x2 float4 gather, 2x2 float4 forward
    (2, 3, 9, 12, 2, 2),          # 2x2 float4 gather, uncovered last row
    (2, 3, 9, 11, 2, 2),          # scalar gather with an uncovered last row / column
    (2, 3, 10, 9, 3, 3),
    (2, 3, 8, 10, 2, 3),          # gaps between windows
    (2, 3, 9, 11, 3, 2),          # overlapping windows: cleared buffer + scatter
])
def test_maxpool_fused_forward_backward(dev, B, C, H, W, p, s):
    rng = np.random.default_rng(H + W + p + s)
    x = _pool_input(rng, B, C, H, W)
    oH, oW = (H - p) // s + 1, (W - p) // s + 1
    n = B * C * oH * oW
    hx = dev.buf(x)
    out, hidx = _fused_forward(dev, hx, B, C, H, W, p, s)
    o, v, idx = S.maxpool_forward(x, B, C, H, W, p, s, oH, oW)
    _same(dev.read(out)[:n], v)
    assert np.array_equal(dev.read(hidx, U32)[:n], idx)
    # overlapping windows can pick one element twice: give every output the same gradient then
    dz = np.full(n, 0.75, np.float32) if s < p else rng.standard_normal(n).astype(np.float32)
    hdz = dev.buf(dz)
    dx = dev.lib.MaxPoolBackwardFused(hdz, hidx, B, C, oH, oW, x.size)
    assert dx, dev.error()
    want = S.maxpool_backward(np.zeros(x.size, np.float32), dz, idx, B, C, oH, oW)
    _same(dev.read(dx)[: x.size], want)
    dev.free(hx, out, hdz, dx)                          # hidx was released by the backward call


def test_maxpool_fused_backward_indices_rewritten(dev):
    """An index buffer rewritten after the forward pass (indices outside their
    own windows) still gives the reference's cleared-buffer-plus-scatter result."""
    B, C, H, W = 2, 2, 8, 8
    rng = np.random.default_rng(9)
    x = rng.standard_normal(B * C * H * W).astype(np.float32)
    hx = dev.buf(x)
    out, hidx = _fused_forward(dev, hx, B, C, H, W, 2, 2)
    n = B * C * 4 * 4
    idx = dev.read(hidx, U32)[:n].copy()
    idx[[1, 17, 40]] = [200, 0, 255]                    # other windows / other planes, distinct targets
    idx[5] = 0xFFFFFFFF
    dev.lib.UpdateBuffer(hidx, idx.view(np.float32).ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    dz = rng.standard_normal(n).astype(np.float32)
    hdz = dev.buf(dz)
    dx = dev.lib.MaxPoolBackwardFused(hdz, hidx, B, C, 4, 4, x.size)
    want = S.maxpool_backward(np.zeros(x.size, np.float32), dz, idx, B, C, 4, 4)
    got = dev.read(dx)[: x.size]
    # 0, 200 and 255 may also be picked by their own windows: either write is the reference's
    for t in (0, 200, 255):
        cands = {float(dz[o]) for o in np.flatnonzero(idx == t)}
        assert float(got[t]) in cands
        got[t] = want[t]
    _same(got, want)
    # the fix-up flag was cleared: a normal forward / backward afterwards is exact
    out2, hidx2 = _fused_forward(dev, hx, B, C, H, W, 2, 2)
    idx2 = dev.read(hidx2, U32)[:n].copy()
    dx2 = dev.lib.MaxPoolBackwardFused(hdz, hidx2, B, C, 4, 4, x.size)
    _same(dev.read(dx2)[: x.size], S.maxpool_backward(np.zeros(x.size, np.float32), dz, idx2, B, C, 4, 4))
    dev.free(hx, out, hdz, dx, out2, dx2)


def test_maxpool_fused_rejects_bad_geometry(dev):
    hx = dev.buf(np.zeros(64, np.float32))
    pidx = ctypes.c_void_p()
    assert not dev.lib.MaxPoolForwardFused(hx, 1, 1, 8, 8, 0, 2, ctypes.byref(pidx))
    assert not dev.lib.MaxPoolForwardFused(hx, 1, 1, 8, 8, 2, 0, ctypes.byref(pidx))
    assert not dev.lib.MaxPoolForwardFused(hx, 1, 1, 1, 8, 2, 2, ctypes.byref(pidx))
    assert not dev.lib.MaxPoolForwardFused(hx, 2, 1, 8, 8, 2, 2, ctypes.byref(pidx))     # x too small
    assert pidx.value is None
    assert dev.error()[0] != 0
    dev.clear_error()
    dev.free(hx)


# ---- conv reshapes ------------------------------------------------------------------------
@pytest.mark.parametrize("B,OC,OH,OW,act,full", [
    (3, 5, 4, 8, 0, True), (3, 5, 4, 8, 1, True), (3, 5, 4, 8, 2, True),     # P % 4 == 0: 128-bit path
    (2, 7, 3, 5, 1, True), (2, 7, 3, 5, 2, True),                            # P = 15: scalar path
    (3, 20, 4, 8, 1, False),
])
def test_conv_reshape(dev, B, OC, OH, OW, act, full):
    rng = np.random.default_rng(OC * 10 + act)
    P = OH * OW
    mm = (3 * rng.standard_normal(OC * B * P)).astype(np.float32)
    mm[::11] = np.nan
    bias = rng.standard_normal(OC).astype(np.float32)
    g = ((B * P + 15) // 16, (OC + 15) // 16, 1) if full else ((B * P + 15) // 16 - 1, 1, 1)
    hm, hb, ho = dev.buf(mm), dev.buf(bias), dev.empty(B * OC * P, fill=-3.0)
    dev.run("conv_reshape", [hm, hb], [ho], g, [B, OC, OH, OW, act])
    want = np.full(B * OC * P, -3.0, np.float32)
    dst, v = S.conv_reshape(mm, bias, B, OC, OH, OW, act, lim_bp=g[0] * 16, lim_oc=g[1] * 16)
    want[dst] = v
    got = dev.read(ho)
    if act == 2:
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan)
        assert ulp_diff(got[~nan], want[~nan]).max() <= 2
    else:
        _same(got, want)
    dev.free(hm, hb, ho)


@pytest.mark.parametrize("B,OC,OH,OW,relu,full", [
    (3, 5, 4, 8, False, True), (3, 5, 4, 8, True, True),
    (2, 7, 3, 5, True, True), (3, 20, 4, 8, True, False),
])
def test_conv_grad_reshape(dev, B, OC, OH, OW, relu, full):
    rng = np.random.default_rng(OC + relu)
    P = OH * OW
    dz = rng.standard_normal(B * OC * P).astype(np.float32)
    fwd = np.maximum(rng.standard_normal(B * OC * P), 0).astype(np.float32)
    fwd[::9] = np.nan
    g = ((B * P + 15) // 16, (OC + 15) // 16, 1) if full else ((B * P + 15) // 16, 1, 1)
    hz, hf, ho = dev.buf(dz), dev.buf(fwd), dev.empty(OC * B * P, fill=2.0)
    name = "conv_grad_reshape_relu" if relu else "conv_grad_reshape"
    dev.run(name, [hz, hf] if relu else [hz], [ho], g, [B, 0, 0, 0, OC, 0, 0, OH, OW])
    want = np.full(OC * B * P, 2.0, np.float32)
    dst, v = S.conv_grad_reshape(dz, B, OC, OH, OW, fwd=fwd if relu else None, lim_bp=g[0] * 16, lim_oc=g[1] * 16)
    want[dst] = v
    _same(dev.read(ho), want)
    dev.free(hz, hf, ho)


def test_layout_shaders_refuse_small_buffers(dev):
    hx, hy = dev.buf(np.zeros(10, np.float32)), dev.empty(100)
    dev.run("upsample", [hx], [hy], (1, 1, 1), [1, 1, 4, 4, 8, 8, 2, 2])      # X holds 10 < 16
    assert dev.error()[0] != 0
    dev.clear_error()
    dev.run("concat_insert", [hy], [hx], (1, 1, 1), [1, 4, 4, 8, 4])          # Out too small
    assert dev.error()[0] != 0
    dev.clear_error()
    dev.free(hx, hy)


def test_layout_refuses_index_space_past_32_bits(dev):
    """The shaders index with 32-bit uint; a dispatch whose index space passes 2^32 is
    refused (DCT_ERR_ARG) and writes nothing."""
    hx, hy = dev.buf(np.arange(64, dtype=np.float32)), dev.empty(64, fill=4.0)
    dev.run("upsample", [hx], [hy], (1, 1, 1), [65536, 65536, 1, 1, 1, 1, 1, 1])
    assert dev.error()[0] == 4                                      # DCT_ERR_ARG
    dev.clear_error()
    dev.run("conv_grad_reshape", [hx], [hy], (1, 1, 1), [65536, 0, 0, 0, 65536, 0, 0, 1, 1])
    assert dev.error()[0] == 4
    dev.clear_error()
    assert np.all(dev.read(hy) == 4.0)
    dev.free(hx, hy)


def test_maxpool_fused_backward_bad_inputs(dev):
    """A dead index handle or a short gradient buffer: a zeroed dInput and an error,
    never an overrun."""
    B, C, H, W = 1, 2, 8, 8
    hx = dev.buf(np.random.default_rng(3).standard_normal(B * C * H * W).astype(np.float32))
    out, hidx = _fused_forward(dev, hx, B, C, H, W, 2, 2)
    small = dev.buf(np.ones(5, np.float32))                          # needs 2*4*4 = 32
    dx = dev.lib.MaxPoolBackwardFused(small, hidx, B, C, 4, 4, B * C * H * W)
    assert dx and dev.error()[0] == 3                                # DCT_ERR_SIZE
    assert np.all(dev.read(dx) == 0.0)
    dev.clear_error()
    dx2 = dev.lib.MaxPoolBackwardFused(out, hidx, B, C, 4, 4, B * C * H * W)   # hidx was released above
    assert dx2 and dev.error()[0] == 2                               # DCT_ERR_HANDLE
    assert np.all(dev.read(dx2) == 0.0)
    dev.clear_error()
    dev.free(hx, out, small, dx, dx2)


def test_layout_sequence_graph_replay_matches_eager(dev):
    """upsample -> concat_insert -> maxpool_forward -> slice as one RunSequence list:
    replayed as a CUDA graph (captured on the second call) it gives the eager bits."""
    import os
    from directcompute_torch_b200._abi import SeqCmd
    lib = dev.lib
    for n in ("upsample", "concat_insert", "maxpool_forward", "slice"):
        lib.CompileShader(n.encode(), "")

    def cmd(name, srvs, uavs, groups, words):
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

    rng = np.random.default_rng(12)
    B, C, H, W = 2, 3, 8, 16
    x = rng.standard_normal(B * C * H * W).astype(np.float32)
    z = rng.standard_normal(B * C * 4 * H * W).astype(np.float32)
    outs = {}
    for graph in (False, True):
        h = {"x": dev.buf(x), "z": dev.buf(z), "u": dev.empty(B * C * 4 * H * W), "cat": dev.empty(2 * B * C * 4 * H * W),
             "po": dev.empty(2 * B * C * H * W), "pi": dev.empty(2 * B * C * H * W), "sl": dev.empty(B * C * 4 * H * W)}
        S_ = 4 * H * W
        cmds = [
            cmd("upsample", [h["x"]], [h["u"]], ((B * C * S_ + 255) // 256, 1, 1), [B, C, H, W, 2 * H, 2 * W, 2, 2]),
            cmd("concat_insert", [h["u"]], [h["cat"]], ((B * C * S_ + 255) // 256, 1, 1), [B, C, S_, 2 * C, 0]),
            cmd("concat_insert", [h["z"]], [h["cat"]], ((B * C * S_ + 255) // 256, 1, 1), [B, C, S_, 2 * C, C]),
            cmd("maxpool_forward", [h["cat"]], [h["po"], h["pi"]], ((W + 15) // 16, (H + 15) // 16, 2 * B * C),
                [B, 2 * C, 2 * H, 2 * W, 2, 2, H, W]),
            cmd("slice", [h["cat"]], [h["sl"]], ((B * C * S_ + 255) // 256, 1, 1), [B, C, S_, 2 * C, C]),
        ]
        arr = (SeqCmd * len(cmds))(*cmds)
        os.environ["DCT_SEQ_GRAPH"] = "1" if graph else "0"
        try:
            for _ in range(4):
                lib.RunSequence(ctypes.cast(arr, ctypes.c_void_p), len(cmds))
            dev.sync()
        finally:
            os.environ.pop("DCT_SEQ_GRAPH", None)
        outs[graph] = {k: dev.read(v) for k, v in h.items()}
        dev.free(*h.values())
    for k in outs[False]:
        assert np.array_equal(outs[True][k].view(np.uint32), outs[False][k].view(np.uint32)), k
    u = S.upsample(x, B, C, H, W, 2 * H, 2 * W, 2, 2)
    assert np.array_equal(outs[True]["sl"], z)
    cat = np.empty(2 * B * C * 4 * H * W, np.float32)
    S.concat_insert(cat, u, B, C, 4 * H * W, 2 * C, 0)
    S.concat_insert(cat, z, B, C, 4 * H * W, 2 * C, C)
    _, v, i = S.maxpool_forward(cat, B, 2 * C, 2 * H, 2 * W, 2, 2, H, W)
    assert np.array_equal(outs[True]["po"], v) and np.array_equal(outs[True]["pi"].view(np.uint32), i)
