"""Pin the layout oracle (upsample, channel concat / slice, max pooling, conv reshapes) on CPU.

The reference checks these ops against PyTorch only inside its UNet comparison:
verify_unet.py:123-132 runs F.max_pool2d(., 2), F.interpolate(scale 2,
nearest) and torch.cat(dim=1) where verify_unet.py:176-182 runs
dc.maxpool2d / dc.upsample2d / dc.concat.  The same comparison runs here,
forward and backward, first through the reference's own nn_engine.py over
oracle.fakelib (its Functions, its cbuffer packing, MaxPool*Fused as
engine.cpp:880-929 does it), then on the oracle functions directly, with
uneven scales, ragged pooling edges and overlapping windows added.
Layout results are bit-exact; only the softmax-CE head and tanh carry a
tolerance.
"""
import numpy as np
import pytest

from oracle import shaders as S
from oracle.newops import ulp_diff

torch = pytest.importorskip("torch")
F = torch.nn.functional


def _t(a, grad=False):
    return torch.tensor(np.asarray(a), dtype=torch.float32, requires_grad=grad)


@pytest.fixture(scope="module")
def nn(reference_dir):
    from oracle.fakelib import FakeLib, load_reference_engine
    return load_reference_engine(reference_dir, FakeLib())


def test_unet_layout_chain_matches_pytorch(nn):
    """maxpool -> upsample -> concat -> global pool -> softmax-CE, as verify_unet.py does it."""
    rng = np.random.default_rng(7)
    x_np = rng.standard_normal((2, 3, 8, 12)).astype(np.float32)
    lab = rng.integers(0, 6, 2)
    x = nn.Tensor(x_np, requires_grad=True)
    p = nn.maxpool2d(x, 2, 2)
    u = nn.upsample2d(p, 2, 2)
    c = nn.concat([u, x], axis=1)
    loss = nn.softmax_ce(nn.global_avg_pool2d(c), nn.Tensor(lab.astype(np.float32)))
    loss.backward()

    xt = _t(x_np, True)
    pt = F.max_pool2d(xt, 2)
    ut = F.interpolate(pt, scale_factor=2, mode="nearest")
    ct = torch.cat([ut, xt], 1)
    lt = F.cross_entropy(ct.mean(dim=(2, 3)), torch.tensor(lab))
    lt.backward()

    assert np.array_equal(p.sync().reshape(pt.shape), pt.detach().numpy())
    assert np.array_equal(u.sync().reshape(ut.shape), ut.detach().numpy())
    assert np.array_equal(c.sync().reshape(ct.shape), ct.detach().numpy())
    assert abs(float(loss.sync()[0]) - float(lt)) < 1e-6
    np.testing.assert_allclose(x.grad.sync().reshape(x_np.shape), xt.grad.numpy(), rtol=1e-5, atol=1e-8)


@pytest.mark.parametrize("sH,sW", [(2, 2), (3, 2), (1, 4)])
def test_upsample_matches_interpolate(sH, sW):
    rng = np.random.default_rng(sH * 10 + sW)
    B, C, H, W = 2, 3, 5, 7
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    out = S.upsample(x.ravel(), B, C, H, W, H * sH, W * sW, sH, sW)
    xt = _t(x, True)
    yt = F.interpolate(xt, size=(H * sH, W * sW), mode="nearest")
    assert np.array_equal(out.reshape(yt.shape), yt.detach().numpy())
    dy = rng.standard_normal(yt.shape).astype(np.float32)
    yt.backward(_t(dy))
    dx = S.upsample_backward(dy.ravel(), B, C, H, W, H * sH, W * sW, sH, sW)
    np.testing.assert_allclose(dx.reshape(x.shape), xt.grad.numpy(), rtol=2e-7, atol=0)


def test_upsample_backward_skips_positions_past_the_output():
    # outH/outW smaller than in*scale: the HLSL bounds check drops the tail of each block
    dy = np.arange(1, 1 + 5 * 7, dtype=np.float32)
    dx = S.upsample_backward(dy, 1, 1, 3, 4, 5, 7, 2, 2)
    full = np.zeros((6, 8), np.float32)
    full[:5, :7] = dy.reshape(5, 7)
    want = full.reshape(3, 2, 4, 2).sum(axis=(1, 3))
    assert np.array_equal(dx.reshape(3, 4), want)


def test_concat_and_slice_match_torch():
    rng = np.random.default_rng(3)
    a = rng.standard_normal((2, 3, 4, 5)).astype(np.float32)
    b = rng.standard_normal((2, 4, 4, 5)).astype(np.float32)
    out = np.full(2 * 7 * 20, np.nan, np.float32)
    S.concat_insert(out, a.ravel(), 2, 3, 20, 7, 0)
    S.concat_insert(out, b.ravel(), 2, 4, 20, 7, 3)
    assert np.array_equal(out.reshape(2, 7, 4, 5), torch.cat([_t(a), _t(b)], 1).numpy())
    assert np.array_equal(S.slice_channels(out, 2, 4, 20, 7, 3).reshape(b.shape), b)
    assert np.array_equal(S.slice_channels(out, 2, 3, 20, 7, 0).reshape(a.shape), a)


@pytest.mark.parametrize("p,s,H,W", [(2, 2, 8, 12), (2, 2, 9, 11), (3, 3, 10, 9), (3, 2, 9, 11), (2, 3, 8, 10)])
def test_maxpool_matches_max_pool2d(p, s, H, W):
    rng = np.random.default_rng(p * 100 + s * 10 + H)
    B, C = 2, 3
    x = rng.standard_normal((B, C, H, W)).astype(np.float32)
    oH, oW = (H - p) // s + 1, (W - p) // s + 1
    o, v, idx = S.maxpool_forward(x.ravel(), B, C, H, W, p, s, oH, oW)
    xt = _t(x, True)
    yt, it = F.max_pool2d(xt, p, s, return_indices=True)
    assert np.array_equal(o, np.arange(B * C * oH * oW))
    assert np.array_equal(v.reshape(yt.shape), yt.detach().numpy())
    plane = (np.arange(B * C) * H * W).repeat(oH * oW)
    assert np.array_equal(idx.astype(np.int64) - plane, it.numpy().ravel())
    if s >= p:              # windows do not overlap: the scatter has one writer per element
        dz = rng.standard_normal(yt.shape).astype(np.float32)
        yt.backward(_t(dz))
        dx = S.maxpool_backward(np.zeros(x.size, np.float32), dz.ravel(), idx, B, C, oH, oW)
        assert np.array_equal(dx.reshape(x.shape), xt.grad.numpy())


def test_maxpool_sentinel_and_nan():
    x = np.array([[-np.inf, np.nan], [np.float32(-2e30), np.nan]], np.float32).ravel()
    _, v, idx = S.maxpool_forward(x, 1, 1, 2, 2, 2, 2, 1, 1)
    assert v[0] == np.float32(-1e30) and idx[0] == 0xFFFFFFFF
    x2 = np.array([np.nan, 1.0, 1.0, 0.5], np.float32)          # NaN skipped, first of the ties wins
    _, v, idx = S.maxpool_forward(x2, 1, 1, 2, 2, 2, 2, 1, 1)
    assert v[0] == 1.0 and idx[0] == 1
    d = np.full(4, 7.0, np.float32)
    S.maxpool_backward(d, np.array([3.0], np.float32), np.array([0xFFFFFFFF], np.uint32), 1, 1, 1, 1)
    assert np.all(d == 7.0)                                      # no index -> no write


@pytest.mark.parametrize("act", [0, 1, 2])
def test_conv_reshape_matches_permute(act):
    rng = np.random.default_rng(act)
    B, OC, OH, OW = 3, 5, 4, 6
    P = OH * OW
    mm = (3 * rng.standard_normal((OC, B * P))).astype(np.float32)
    bias = rng.standard_normal(OC).astype(np.float32)
    dst, v = S.conv_reshape(mm.ravel(), bias, B, OC, OH, OW, act)
    out = np.empty(B * OC * P, np.float32)
    out[dst] = v
    z = _t(mm).reshape(OC, B, P).permute(1, 0, 2) + _t(bias)[None, :, None]
    want = {0: z, 1: torch.relu(z), 2: torch.tanh(z)}[act].numpy().ravel()
    if act == 2:                                                 # tanh: float64-rounded vs torch's float32
        assert ulp_diff(out, want).max() <= 2
    else:
        assert np.array_equal(out, want)


@pytest.mark.parametrize("relu", [False, True])
def test_conv_grad_reshape_matches_permute(relu):
    rng = np.random.default_rng(11 + relu)
    B, OC, OH, OW = 3, 5, 4, 6
    P = OH * OW
    dz = rng.standard_normal((B, OC, P)).astype(np.float32)
    fwd = np.maximum(rng.standard_normal((B, OC, P)), 0).astype(np.float32) if relu else None
    if relu:
        fwd.ravel()[::7] = np.nan                                   # NaN keeps the gradient
    dst, v = S.conv_grad_reshape(dz.ravel(), B, OC, OH, OW, fwd=None if fwd is None else fwd.ravel())
    out = np.empty(OC * B * P, np.float32)
    out[dst] = v
    g = dz if not relu else np.where(fwd <= 0, 0, dz).astype(np.float32)
    assert np.array_equal(out, g.transpose(1, 0, 2).ravel())
