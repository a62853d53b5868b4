"""The reference's Python API (directcompute_torch_b200.engine) on the GPU, against PyTorch.

The reference verifies its engine against PyTorch: verify_unet.py:123-132 /
:176-182 (max pool, nearest upsample, channel concat), verify_batchnorm.py:6-64
(BatchNorm2d forward and backward) and nn_verify.py's softmax / grad checks.
The same comparisons run here through engine.py's Functions and autograd tape,
which dispatch libdct_cuda.so's kernels with the reference's cbuffer words.
Layout results are bit-exact; losses and gradients through softmax-CE and
BatchNorm are held to rel 1e-5.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
F = torch.nn.functional


@pytest.fixture(scope="module")
def E():
    from directcompute_torch_b200 import engine
    return engine


def _t(a, grad=False):
    return torch.tensor(np.asarray(a), dtype=torch.float32, requires_grad=grad)


def test_unet_layout_chain(E):
    """maxpool -> upsample -> concat -> global pool -> softmax-CE, forward and backward."""
    rng = np.random.default_rng(21)
    x_np = rng.standard_normal((2, 3, 16, 24)).astype(np.float32)
    lab = rng.integers(0, 6, 2)
    x = E.Tensor(x_np, requires_grad=True)
    p = E.maxpool2d(x, 2, 2)
    u = E.upsample2d(p, 2, 2)
    c = E.concat([u, x], axis=1)
    loss = E.softmax_ce(E.global_avg_pool2d(c), E.Tensor(lab.astype(np.float32)))
    loss.backward()

    xt = _t(x_np, True)
    pt = F.max_pool2d(xt, 2)
    ut = F.interpolate(pt, scale_factor=2, mode="nearest")
    ct = torch.cat([ut, xt], 1)
    lt = F.cross_entropy(ct.mean(dim=(2, 3)), torch.tensor(lab))
    lt.backward()

    assert np.array_equal(p.sync(), pt.detach().numpy())
    assert np.array_equal(u.sync(), ut.detach().numpy())
    assert np.array_equal(c.sync(), ct.detach().numpy())
    assert abs(float(loss.sync()[0]) - float(lt.detach())) <= 1e-5 * abs(float(lt.detach()))
    np.testing.assert_allclose(x.grad.sync(), xt.grad.numpy(), rtol=1e-5, atol=1e-9)


def test_uneven_upsample_and_overlapping_pool(E):
    rng = np.random.default_rng(22)
    x_np = rng.standard_normal((2, 2, 5, 7)).astype(np.float32)
    x = E.Tensor(x_np, requires_grad=True)
    u = E.upsample2d(x, 3, 2)                       # [2, 2, 15, 14]
    m = E.maxpool2d(u, 3, 2)                        # overlapping windows
    out = m.sync()
    xt = _t(x_np, True)
    ut = F.interpolate(xt, size=(15, 14), mode="nearest")
    mt = F.max_pool2d(ut, 3, 2)
    assert np.array_equal(u.sync(), ut.detach().numpy())
    assert np.array_equal(out, mt.detach().numpy())
    # the upsample gradient alone (the pool's overlapping windows leave ties to the scatter order)
    g_np = rng.standard_normal(u.shape).astype(np.float32)
    u._ctx.backward(E.Tensor(g_np))
    ut.backward(_t(g_np))
    np.testing.assert_allclose(x.grad.sync(), xt.grad.numpy(), rtol=2e-7, atol=0)


def test_dense_head_softmax_ce(E):
    rng = np.random.default_rng(23)
    B, K = 64, 10
    x_np = (2 * rng.standard_normal((B, K))).astype(np.float32)
    b_np = (0.1 * rng.standard_normal(K)).astype(np.float32)
    lab = rng.integers(0, K, B)
    x = E.Tensor(x_np, requires_grad=True)
    b = E.Tensor(b_np, requires_grad=True)
    loss = E.softmax_ce(E.bias_relu(x, b), E.Tensor(lab.astype(np.float32)))
    loss.backward()
    xt, bt = _t(x_np, True), _t(b_np, True)
    lt = F.cross_entropy(torch.relu(xt + bt), torch.tensor(lab))
    lt.backward()
    assert abs(float(loss.sync()[0]) - float(lt.detach())) <= 1e-5 * abs(float(lt.detach()))
    np.testing.assert_allclose(x.grad.sync(), xt.grad.numpy(), rtol=1e-5, atol=1e-8)
    np.testing.assert_allclose(b.grad.sync(), bt.grad.numpy(), rtol=1e-5, atol=1e-8)


def test_batchnorm2d_train_forward_backward(E):
    rng = np.random.default_rng(24)
    x_np = (0.5 + 2 * rng.standard_normal((8, 4, 6, 6))).astype(np.float32)
    lab = rng.integers(0, 4, 8)
    x = E.Tensor(x_np, requires_grad=True)
    bn = E.BatchNorm2d(4)
    y = bn(x)
    loss = E.softmax_ce(E.global_avg_pool2d(y), E.Tensor(lab.astype(np.float32)))
    loss.backward()
    xt = _t(x_np, True)
    btn = torch.nn.BatchNorm2d(4, eps=1e-5, momentum=0.1)
    yt = btn(xt)
    lt = F.cross_entropy(yt.mean(dim=(2, 3)), torch.tensor(lab))
    lt.backward()
    np.testing.assert_allclose(y.sync(), yt.detach().numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(x.grad.sync(), xt.grad.numpy(), rtol=1e-4, atol=1e-7)
    np.testing.assert_allclose(bn.running_mean.sync(), btn.running_mean.numpy(), rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(bn.running_var.sync(), btn.running_var.numpy(), rtol=1e-5, atol=1e-7)
