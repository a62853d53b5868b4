"""Pin the oracle against the reference's OWN checks (CPU, no GPU).

The reference publishes no golden vectors; its known-answer tests for this path
are nn_verify.py (verify_relu :300-315, verify_softmax :318-342, verify_linear
:424-446, grad_check :63-142), verify_batchnorm.py:6-64 (against PyTorch) and
verify_dice_loss.py:17-60.  Each runs here UNMODIFIED, with the reference's
`nn_engine.py` bound to `oracle.fakelib.FakeLib` in place of engine.dll.
"""
import contextlib
import importlib
import io
import sys

import numpy as np
import pytest

from oracle.fakelib import FakeLib, load_reference_engine


@pytest.fixture(scope="module")
def ref(reference_dir):
    fl = FakeLib()
    nn = load_reference_engine(reference_dir, fl)
    sys.modules.pop("nn_verify", None)
    nv = importlib.import_module("nn_verify")
    return nn, nv, fl


def test_engine_binds_every_symbol(ref):
    nn, _, fl = ref
    assert nn.lib is fl
    # nn_engine.py compiled its 69 shader names (plus matmul_dgpu for a dGPU)
    assert len(fl._compiled) >= 69


def test_verify_relu(ref):
    _, nv, _ = ref
    np.random.seed(42)
    ok, err = nv.verify_relu(N=4099, verbose=False)
    assert ok and err == 0.0


def test_verify_softmax(ref):
    _, nv, _ = ref
    np.random.seed(42)
    ok, rel = nv.verify_softmax(batch=33, classes=1000, verbose=False)
    assert ok and rel < 1e-6


def test_verify_linear_exercises_add_bias(ref):
    _, nv, _ = ref
    np.random.seed(42)
    ok, rel = nv.verify_linear(in_f=64, out_f=48, batch=16, verbose=False)
    assert ok


@pytest.mark.parametrize("fn", ["softmax_ce_bias", "bias_relu"])
def test_grad_check(ref, fn):
    nn, nv, _ = ref
    np.random.seed(0)
    x = nn.Tensor(np.random.randn(8, 12).astype(np.float32), requires_grad=True, track=False)
    w = nn.Tensor((np.random.randn(12, 6) * 0.5).astype(np.float32), requires_grad=True, track=False)
    b = nn.Tensor((np.random.randn(6) * 0.5).astype(np.float32), requires_grad=True, track=False)
    y = nn.Tensor(np.arange(8, dtype=np.float32) % 6, track=False)
    act = nn.add_bias if fn == "softmax_ce_bias" else nn.bias_relu
    ok, rel, _ = nv.grad_check(lambda: nn.softmax_ce(act(nn.matmul(x, w), b), y), b, verbose=False)
    assert ok, rel


def test_verify_batchnorm_against_pytorch(ref, reference_dir):
    pytest.importorskip("torch")
    sys.modules.pop("verify_batchnorm", None)
    vb = importlib.import_module("verify_batchnorm")
    with contextlib.redirect_stdout(io.StringIO()):
        vb.test_batchnorm()          # asserts y < 1e-4, dx/dgamma/dbeta < 1e-3 internally


def test_verify_dice_loss(ref):
    sys.modules.pop("verify_dice_loss", None)
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        importlib.import_module("verify_dice_loss")
    out = buf.getvalue()
    assert out.count("PASSED") == 2 and "FAILED" not in out, out
