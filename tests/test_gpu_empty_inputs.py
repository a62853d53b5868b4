"""Empty operands through the C-ABI: NumPy's results, and the reference's for an empty batch.

- `dct_unary` over 0 elements, and `dct_binary` with a zero-length dimension, write
  nothing and succeed. NumPy returns an empty array.
- `dct_reduce` over a zero-length axis gives 0 for sum and NaN for mean, as
  `np.sum` / `np.mean` of an empty axis do. max, min, argmax and argmin fail with
  DCT_ERR_ARG and write nothing, since NumPy raises. With an empty outer or inner
  extent the output is empty and nothing is written.
- `dct_reduce_all` of an empty vector: sum 0, mean NaN, max an error.
- The reference's `loss` shader with batch_size 0 writes 0 / 0 = NaN
  (nn_loss.hlsl:41), and so does the library's `loss`. `dct_softmax_ce` over 0 rows
  gives NaN with the default divisor, and 0 with a global divisor: the case of a
  rank that holds no rows of a sharded batch.
"""
import warnings

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_unary_and_binary_over_nothing(dev):
    x, y = dev.empty(8, fill=3.0), dev.empty(8, fill=7.0)
    dev.unary("exp", x, y, 0)
    assert (dev.read(y) == 7.0).all()
    a, b, out = dev.empty(4, fill=1.0), dev.empty(4, fill=2.0), dev.empty(8, fill=7.0)
    assert np.add(np.ones((0, 4), np.float32), np.ones((1, 4), np.float32)).shape == (0, 4)
    dev.binary("add", a, [0, 4], b, [1, 4], out)
    dev.binary("mul", a, [3, 0], b, [1], out)
    assert (dev.read(out) == 7.0).all()
    assert dev.error()[0] == 0
    dev.free(x, y, a, b, out)


def test_reduce_over_an_empty_axis(dev):
    x = dev.empty(4, fill=1.0)
    out = dev.empty(12, fill=7.0)
    empty = np.zeros((3, 0, 4), np.float32)
    dev.reduce("sum", x, 3, 0, 4, out)
    got = dev.read(out)
    assert np.array_equal(got, np.sum(empty, axis=1).ravel()) and not np.signbit(got).any()
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", RuntimeWarning)               # NumPy: "Mean of empty slice"
        want = np.mean(empty, axis=1).ravel()
    dev.reduce("mean", x, 3, 0, 4, out)
    assert np.isnan(want).all() and np.isnan(dev.read(out)).all()
    for op in ("max", "min", "argmax", "argmin"):
        with pytest.raises(ValueError):
            getattr(np, op)(empty, axis=1)
        with pytest.raises(RuntimeError, match="ARG.*zero-length axis"):
            dev.reduce(op, x, 3, 0, 4, out)
        assert np.isnan(dev.read(out)).all(), op              # nothing written
    dev.clear_error()
    # an empty output (outer or inner 0): nothing to write, no error
    out2 = dev.empty(4, fill=5.0)
    dev.reduce("max", x, 0, 4, 1, out2)
    dev.reduce("sum", x, 1, 4, 0, out2)
    assert (dev.read(out2) == 5.0).all()
    dev.free(x, out, out2)


def test_reduce_all_of_an_empty_vector(dev):
    x, out = dev.empty(4, fill=1.0), dev.empty(1, fill=7.0)
    assert dev.reduce_all("sum", x, 0, out) == 0.0 and dev.read(out)[0] == 0.0
    v = dev.reduce_all("mean", x, 0, out)
    assert np.isnan(v) and np.isnan(dev.read(out)[0])
    with pytest.raises(RuntimeError, match="ARG.*empty vector"):
        dev.reduce_all("max", x, 0, out)
    dev.clear_error()
    dev.free(x, out)


def test_empty_batch_loss(dev):
    K = 10
    logits, labels = dev.empty(K, fill=0.5), dev.empty(1, fill=3.0)
    loss = dev.empty(1, fill=7.0)
    # the reference shader: partial[0] / (float)batch_size with batch_size 0
    with np.errstate(invalid="ignore"):
        assert np.isnan(np.float32(0.0) / np.float32(0))
    dev.run("loss", [logits, labels], [loss], (1, 1, 1), [0, K, 0, 0])
    assert np.isnan(dev.read(loss)[0])
    lib = dev.lib
    rc = lib.dct_softmax_ce(logits, labels, 0, 0, K, None, None, loss, None, 0.0, 0.0)
    assert rc == 0, dev.error()
    assert np.isnan(dev.read(loss)[0])
    rc = lib.dct_softmax_ce(logits, labels, 0, 0, K, None, None, loss, None, 256.0, 256.0)
    assert rc == 0, dev.error()
    assert dev.read(loss)[0] == 0.0
    dev.free(logits, labels, loss)
