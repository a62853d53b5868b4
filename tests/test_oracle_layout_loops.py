"""The vectorised layout oracle against a literal per-thread restatement of each shader.

Each function below walks the dispatch's thread grid (groups x [numthreads]) the way
the HLSL does -- one SV_DispatchThreadID at a time, the same early returns, the same
index arithmetic in 32-bit `uint` -- for nn_upsample.hlsl, nn_upsample_backward.hlsl,
nn_concat_insert.hlsl, nn_slice.hlsl, nn_maxpool_forward.hlsl, nn_maxpool_backward.hlsl,
nn_conv_reshape.hlsl, nn_conv_grad_reshape.hlsl and nn_conv_grad_reshape_relu.hlsl.
`oracle.shaders.run_shader` must give the same bits on random small dispatches,
including partial group counts and ragged shapes.
"""
import struct

import numpy as np
import pytest

from oracle import shaders as S

F32 = np.float32
M32 = 0xFFFFFFFF


def _cb(*w):
    return struct.pack("<%dI" % len(w), *[int(v) & M32 for v in w])


def _threads_1d(groups, tpg=256):
    return range(groups[0] * tpg)


def loop_upsample(X, Out, u, groups):
    B, C, inH, inW, oH, oW, sH, sW = u
    total = (B * C * oH * oW) & M32
    for i in _threads_1d(groups):
        if i >= total:
            continue
        w = i % oW; t = i // oW; h = t % oH; t //= oH; c = t % C; b = t // C
        Out[i] = X[((b * C + c) * inH + h // sH) * inW + w // sW]


def loop_upsample_backward(DY, DX, u, groups):
    B, C, inH, inW, oH, oW, sH, sW = u
    total = (B * C * inH * inW) & M32
    for i in _threads_1d(groups):
        if i >= total:
            continue
        w = i % inW; t = i // inW; h = t % inH; t //= inH; c = t % C; b = t // C
        s = F32(0.0)
        for sh in range(sH):
            for sw in range(sW):
                ho, wo = h * sH + sh, w * sW + sw
                if ho < oH and wo < oW:
                    s = F32(s + DY[((b * C + c) * oH + ho) * oW + wo])
        DX[i] = s


def loop_concat(X, Out, u, groups):
    B, cin, Sp, cout, coff = u
    total = B * cin * Sp
    for i in _threads_1d(groups):
        if i >= total:
            continue
        s = i % Sp; t = i // Sp; c = t % cin; b = t // cin
        Out[(b * cout + c + coff) * Sp + s] = X[i]


def loop_slice(DY, DX, u, groups):
    B, cin, Sp, cout, coff = u
    total = B * cin * Sp
    for i in _threads_1d(groups):
        if i >= total:
            continue
        s = i % Sp; t = i // Sp; c = t % cin; b = t // cin
        DX[i] = DY[(b * cout + c + coff) * Sp + s]


def loop_maxpool_forward(X, Out, Idx, u, groups):
    B, C, inH, inW, p, st, oH, oW = u
    for bc in range(groups[2]):
        for oh in range(groups[1] * 16):
            for ow in range(groups[0] * 16):
                if ow >= oW or oh >= oH or bc >= B * C:
                    continue
                best, bi = F32(-1e30), M32
                base = bc * inH * inW
                for ph in range(p):
                    for pw in range(p):
                        ih, iw = oh * st + ph, ow * st + pw
                        if ih < inH and iw < inW:
                            k = base + ih * inW + iw
                            if X[k] > best:
                                best, bi = X[k], k
                o = bc * oH * oW + oh * oW + ow
                Out[o] = best
                Idx[o] = bi


def loop_maxpool_backward(DZ, Idx, DI, u, groups):
    B, C, oH, oW = u
    for bc in range(groups[2]):
        for oh in range(groups[1] * 16):
            for ow in range(groups[0] * 16):
                if ow >= oW or oh >= oH or bc >= B * C:
                    continue
                o = bc * oH * oW + oh * oW + ow
                k = int(Idx[o])
                if k != M32 and k < DI.size:              # D3D11 drops writes past the UAV
                    DI[k] = DZ[o]


def loop_conv_reshape(MM, BIAS, Out, u, groups):
    B, OC, OH, OW, act = u
    BP = B * OH * OW
    for oc in range(groups[1] * 16):
        for bp in range(groups[0] * 16):
            if oc >= OC or bp >= BP:
                continue
            z = F32(MM[oc * BP + bp] + BIAS[oc])
            a = (z if z > 0 else F32(0.0)) if act == 1 else (F32(np.tanh(np.float64(z))) if act == 2 else z)
            b, px = bp // (OH * OW), bp % (OH * OW)
            Out[b * OC * OH * OW + oc * OH * OW + px] = a


def loop_conv_grad_reshape(DZ, FWD, Out, u, groups):
    B, OC, OH, OW = u[0], u[4], u[7], u[8]
    BP = B * OH * OW
    for oc in range(groups[1] * 16):
        for bp in range(groups[0] * 16):
            if oc >= OC or bp >= BP:
                continue
            b, px = bp // (OH * OW), bp % (OH * OW)
            src = b * OC * OH * OW + oc * OH * OW + px
            g = DZ[src]
            if FWD is not None and FWD[src] <= 0:
                g = F32(0.0)
            Out[oc * BP + bp] = g


def _bits_equal(a, b):
    a, b = np.asarray(a, F32), np.asarray(b, F32)
    return np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("seed", range(6))
def test_upsample_pair(seed):
    r = np.random.default_rng(seed)
    B, C, inH, inW = (int(v) for v in r.integers(1, 4, 4))
    sH, sW = (int(v) for v in r.integers(1, 4, 2))
    oH, oW = inH * sH - int(r.integers(0, 2)), inW * sW - int(r.integers(0, 2))
    u = [B, C, inH, inW, max(oH, 1), max(oW, 1), sH, sW]
    x = r.standard_normal(B * C * inH * inW + 64).astype(F32)
    total = B * C * u[4] * u[5]
    groups = (max(1, (total + 255) // 256 - int(r.integers(0, 2))), 1, 1)
    want = np.full(total + 8, 3.0, F32); got = want.copy()
    loop_upsample(x, want, u, groups)
    S.run_shader("upsample", [x], [got], groups, _cb(*u))
    assert _bits_equal(got, want)
    dy = r.standard_normal(total).astype(F32)
    dy[::5] = -0.0
    n_in = B * C * inH * inW
    want = np.full(n_in, 7.0, F32); got = want.copy()
    g2 = (max(1, (n_in + 255) // 256), 1, 1)
    loop_upsample_backward(dy, want, u, g2)
    S.run_shader("upsample_backward", [dy], [got], g2, _cb(*u))
    assert _bits_equal(got, want)


@pytest.mark.parametrize("seed", range(6))
def test_concat_slice(seed):
    r = np.random.default_rng(10 + seed)
    B, cin, Sp = (int(v) for v in r.integers(1, 5, 3))
    coff = int(r.integers(0, 3))
    cout = cin + coff + int(r.integers(0, 3))
    u = [B, cin, Sp, cout, coff]
    x = r.standard_normal(B * cin * Sp).astype(F32)
    n_out = B * cout * Sp
    groups = (max(1, (B * cin * Sp + 255) // 256), 1, 1)
    want = np.full(n_out, np.nan, F32); got = want.copy()
    loop_concat(x, want, u, groups)
    S.run_shader("concat_insert", [x], [got], groups, _cb(*u))
    assert _bits_equal(got, want)
    dy = r.standard_normal(n_out).astype(F32)
    want = np.zeros(B * cin * Sp, F32); got = want.copy()
    loop_slice(dy, want, u, groups)
    S.run_shader("slice", [dy], [got], groups, _cb(*u))
    assert _bits_equal(got, want)


@pytest.mark.parametrize("seed", range(8))
def test_maxpool_pair(seed):
    r = np.random.default_rng(20 + seed)
    B, C = (int(v) for v in r.integers(1, 3, 2))
    p, st = int(r.integers(1, 4)), int(r.integers(1, 4))
    inH, inW = (int(v) for v in r.integers(p, p + 20, 2))
    oH, oW = (inH - p) // st + 1, (inW - p) // st + 1
    x = r.standard_normal(B * C * inH * inW).astype(F32)
    x[r.integers(0, x.size, 5)] = np.nan
    x[r.integers(0, x.size, 5)] = -np.inf
    u = [B, C, inH, inW, p, st, oH, oW]
    groups = ((oW + 15) // 16, (oH + 15) // 16, max(1, B * C - int(r.integers(0, 2))))
    n = B * C * oH * oW
    wv = np.full(n, 2.0, F32); wi = np.full(n, 5, np.uint32)
    gv = wv.copy(); gi = wi.copy()
    loop_maxpool_forward(x, wv, wi, u, groups)
    S.run_shader("maxpool_forward", [x], [gv, gi.view(F32)], groups, _cb(*u))
    assert _bits_equal(gv, wv) and np.array_equal(gi, wi)
    dz = r.standard_normal(n).astype(F32)
    idx = wi.copy()
    idx[::7] = x.size + 3                                   # past the UAV: dropped
    want = np.full(x.size, 9.0, F32); got = want.copy()
    ub = [B, C, oH, oW]
    if st >= p:                                             # one writer per element: the order cannot matter
        loop_maxpool_backward(dz, idx, want, ub, groups)
        S.run_shader("maxpool_backward", [dz, idx.view(F32)], [got], groups, _cb(*ub))
        assert _bits_equal(got, want)


@pytest.mark.parametrize("act", [0, 1, 2])
@pytest.mark.parametrize("partial", [False, True])
def test_conv_reshapes(act, partial):
    r = np.random.default_rng(act * 2 + partial)
    B, OC, OH, OW = 2, 5, 3, 5
    BP = B * OH * OW
    mm = (2 * r.standard_normal(OC * BP)).astype(F32)
    mm[::9] = np.nan
    bias = r.standard_normal(OC).astype(F32)
    groups = ((BP + 15) // 16 - (1 if partial else 0) or 1, (OC + 15) // 16, 1)
    u = [B, OC, OH, OW, act]
    want = np.full(B * OC * OH * OW, 4.0, F32); got = want.copy()
    loop_conv_reshape(mm, bias, want, u, groups)
    S.run_shader("conv_reshape", [mm, bias], [got], groups, _cb(*u))
    if act == 2:
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan) and np.array_equal(got[~nan], want[~nan])
    else:
        assert np.array_equal(np.isnan(got), np.isnan(want))
        assert np.array_equal(got[~np.isnan(got)], want[~np.isnan(want)])
    dz = r.standard_normal(B * OC * OH * OW).astype(F32)
    fwd = np.maximum(r.standard_normal(dz.size), 0).astype(F32)
    fwd[::4] = np.nan
    ug = [B, 0, 0, 0, OC, 0, 0, OH, OW]
    for name, f in (("conv_grad_reshape", None), ("conv_grad_reshape_relu", fwd)):
        want = np.full(OC * BP, 6.0, F32); got = want.copy()
        loop_conv_grad_reshape(dz, f, want, ug, groups)
        S.run_shader(name, [dz] + ([f] if f is not None else []), [got], groups, _cb(*ug))
        assert _bits_equal(got, want), name
