"""NumPy-semantics oracle for the hot-path ops the reference has no GPU kernel for.

The reference's only CPU arithmetic for these is NumPy on float32 arrays (its
verification code: nn_verify.py:224-491, verify_dice_loss.py:17-40, and
`clip_grad_norm` at nn_engine.py:1335-1355), so NumPy's float32 ufunc and
reduction semantics define them:

* binary ops (add, sub, mul, div, maximum, minimum) with NumPy's right-aligned
  broadcasting -- bit-exact targets (`np.maximum` propagates NaN);
* unary exp, log(|x|+1), tanh, sigmoid -- float64 evaluation of the same
  float32 expression, rounded; the device is held to <= 2 ulp.  For
  log(|x|+1) the inner `|x| + 1` is the float32 add NumPy performs;
* sum / mean accumulate in float64 (rel 1e-5 target), max / argmax are exact,
  argmax returns the first index of the maximum and NaN counts as the maximum
  (NumPy's rule);
* fused row softmax + cross-entropy (forward and backward), float64 reference.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
F64 = np.float64

BINARY_OPS = ("add", "sub", "mul", "div", "maximum", "minimum")
UNARY_OPS = ("exp", "log_abs1p", "tanh", "sigmoid", "neg", "abs", "relu")
REDUCE_OPS = ("sum", "mean", "max", "argmax", "min", "argmin")


def binary(op: str, a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """np.add / subtract / multiply / divide / maximum / minimum in float32."""
    a = np.asarray(a, dtype=F32)
    b = np.asarray(b, dtype=F32)
    with np.errstate(all="ignore"):
        if op == "add":
            return np.add(a, b)
        if op == "sub":
            return np.subtract(a, b)
        if op == "mul":
            return np.multiply(a, b)
        if op == "div":
            return np.divide(a, b)
        if op == "maximum":
            return np.maximum(a, b)
        if op == "minimum":
            return np.minimum(a, b)
    raise ValueError(op)


def binary_grads(op: str, a: np.ndarray, b: np.ndarray, g: np.ndarray):
    """Gradients of `binary(op, a, b)` w.r.t. a and b: broadcast grad = sum over expanded dims.

    Returned in float64 (the device accumulates the sums in float64 and rounds).
    maximum/minimum route the gradient to `a` on ties, like NumPy's `a >= b` choice.
    """
    a64, b64, g64 = (np.asarray(t, dtype=F64) for t in (a, b, g))
    with np.errstate(all="ignore"):
        if op == "add":
            ga, gb = g64, g64
        elif op == "sub":
            ga, gb = g64, -g64
        elif op == "mul":
            ga = g64 * np.asarray(np.broadcast_to(b, g.shape), dtype=F32).astype(F64)
            gb = g64 * np.asarray(np.broadcast_to(a, g.shape), dtype=F32).astype(F64)
        elif op == "div":
            bb = np.broadcast_to(b64, g.shape)
            ga = g64 / bb
            gb = -g64 * np.broadcast_to(a64, g.shape) / (bb * bb)
        elif op in ("maximum", "minimum"):
            aa = np.broadcast_to(a, g.shape)
            bb = np.broadcast_to(b, g.shape)
            pick_a = (aa >= bb) if op == "maximum" else (aa <= bb)
            pick_a = pick_a | np.isnan(aa)
            ga = np.where(pick_a, g64, 0.0)
            gb = np.where(pick_a, 0.0, g64)
        else:
            raise ValueError(op)
    return sum_to_shape(np.broadcast_to(ga, g.shape), a.shape), sum_to_shape(np.broadcast_to(gb, g.shape), b.shape)


def sum_to_shape(g: np.ndarray, shape) -> np.ndarray:
    """Reduce a broadcast result back to `shape` (float64 sums over the expanded dims)."""
    g = np.asarray(g, dtype=F64)
    shape = tuple(shape)
    lead = g.ndim - len(shape)
    if lead:
        g = g.sum(axis=tuple(range(lead)))
    axes = tuple(i for i, s in enumerate(shape) if s == 1 and g.shape[i] != 1)
    if axes:
        g = g.sum(axis=axes, keepdims=True)
    return g.reshape(shape)


def unary_f64(op: str, x: np.ndarray) -> np.ndarray:
    """Correctly rounded float32 reference of each unary op (float64 evaluation)."""
    x = np.asarray(x, dtype=F32)
    with np.errstate(all="ignore"):
        if op == "exp":
            return np.exp(x.astype(F64)).astype(F32)
        if op == "log_abs1p":
            t = (np.abs(x) + F32(1.0)).astype(F32)          # NumPy's float32 add
            return np.log(t.astype(F64)).astype(F32)
        if op == "tanh":
            return np.tanh(x.astype(F64)).astype(F32)
        if op == "sigmoid":
            return (1.0 / (1.0 + np.exp(-x.astype(F64)))).astype(F32)
        if op == "neg":
            return -x
        if op == "abs":
            return np.abs(x)
        if op == "relu":
            return np.where(x > 0, x, F32(0.0)).astype(F32)
    raise ValueError(op)


def unary_np32(op: str, x: np.ndarray) -> np.ndarray:
    """The same ops evaluated by NumPy in float32 (the reference's CPU path; timed)."""
    x = np.asarray(x, dtype=F32)
    with np.errstate(all="ignore"):
        if op == "exp":
            return np.exp(x)
        if op == "log_abs1p":
            return np.log(np.abs(x) + F32(1.0))
        if op == "tanh":
            return np.tanh(x)
        if op == "sigmoid":
            return F32(1.0) / (F32(1.0) + np.exp(-x))
        if op == "neg":
            return -x
        if op == "abs":
            return np.abs(x)
        if op == "relu":
            return np.where(x > 0, x, F32(0.0)).astype(F32)
    raise ValueError(op)


def reduce(op: str, x: np.ndarray, axis):
    """NumPy reduction semantics; sums/means from float64 accumulation, rounded once."""
    x = np.asarray(x, dtype=F32)
    if op == "sum":
        return np.sum(x.astype(F64), axis=axis).astype(F32)
    if op == "mean":
        return np.mean(x.astype(F64), axis=axis).astype(F32)
    if op == "max":
        return np.max(x, axis=axis)
    if op == "min":
        return np.min(x, axis=axis)
    if op == "argmax":
        return np.argmax(x, axis=axis).astype(np.int32)
    if op == "argmin":
        return np.argmin(x, axis=axis).astype(np.int32)
    raise ValueError(op)


def full_sum_f64(x: np.ndarray) -> float:
    """Float64-accumulated sum of a flat float32 vector."""
    return float(np.sum(np.asarray(x, dtype=F32).astype(F64)))


def softmax_ce_f64(logits: np.ndarray, labels: np.ndarray, loss_divisor=None):
    """Fused row softmax + mean cross-entropy (float64 reference).

    Returns (probs fp32, loss fp32, logprobs fp32).  `labels` are integer class
    ids (the reference stores them as float, nn_loss.hlsl:16); the divisor is the
    global batch (it differs from the local rows when rows are sharded).
    """
    X = np.asarray(logits, dtype=F32).astype(F64)
    B, K = X.shape
    lab = np.asarray(labels).astype(np.int64)
    mx = X.max(axis=1, keepdims=True)
    z = X - mx
    lse = np.log(np.exp(z).sum(axis=1, keepdims=True))
    logp = z - lse
    p = np.exp(logp)
    div = B if loss_divisor is None else loss_divisor
    loss = -(logp[np.arange(B), lab]).sum() / div
    return p.astype(F32), F32(loss), logp.astype(F32)


def softmax_ce_rows_f64(logits: np.ndarray, labels: np.ndarray):
    """Row-wise form of `softmax_ce_f64` for chunked checks of large batches.

    Returns (probs fp32, per-row cross-entropy float64, logprobs fp32); the mean
    loss of a batch is the float64 sum of the row losses over the global divisor.
    """
    X = np.asarray(logits, dtype=F32).astype(F64)
    B = X.shape[0]
    lab = np.asarray(labels).astype(np.int64)
    z = X - X.max(axis=1, keepdims=True)
    logp = z - np.log(np.exp(z).sum(axis=1, keepdims=True))
    return np.exp(logp).astype(F32), -logp[np.arange(B), lab], logp.astype(F32)


def softmax_ce_dlogits(p_dev: np.ndarray, labels: np.ndarray, divisor: int) -> np.ndarray:
    """dlogits = (p - onehot) / divisor in fp32 from the device's own probs (bit-exact target)."""
    p = np.asarray(p_dev, dtype=F32)
    B, K = p.shape
    onehot = np.zeros((B, K), dtype=F32)
    onehot[np.arange(B), np.asarray(labels).astype(np.int64)] = 1.0
    return ((p - onehot) / F32(divisor)).astype(F32)


def ulp_diff(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in units-in-the-last-place between two float32 arrays (NaN==NaN -> 0)."""
    a = np.ascontiguousarray(a, dtype=F32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, dtype=F32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, np.int64(-2 ** 31) - a, a)
    b = np.where(b < 0, np.int64(-2 ** 31) - b, b)
    return np.abs(a - b)
