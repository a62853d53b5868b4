"""NumPy-semantics ops the reference has no GPU kernel for, with autograd.

The reference's tensor math beyond its fixed shaders lives on its NumPy side
(its checks in nn_verify.py:224-491 and verify_dice_loss.py:17-40, and
`clip_grad_norm` at nn_engine.py:1335-1355), so NumPy's float32 semantics
define these ops.  They run on the library's dct_* entry points:

* broadcast binary ops `add sub mul div maximum minimum` with NumPy's
  right-aligned broadcasting, bit-exact against NumPy float32;
* the broadcast gradient: the upstream gradient summed over the dims an
  operand was broadcast along (`sum_to_shape`, float64 accumulation rounded
  once); maximum/minimum route the gradient to `a` on ties and where `a` is
  NaN;
* unary `exp log_abs1p tanh sigmoid neg abs` (<= 2 ulp against float64 for
  the transcendentals) with fused backward kernels;
* reductions `sum mean max min argmax argmin` over one axis or all of them
  (float64 accumulation; first index on ties; NaN is the maximum); `sum` and
  `mean` are differentiable;
* `softmax_cross_entropy`: the fused row softmax + mean cross-entropy; its
  forward pass also writes dlogits, so the backward is one scaled copy;
* `bias_relu` (the reference's bias_relu shader, nn_bias_relu.hlsl:8-12) whose
  backward is one fused pass (dct_bias_relu_backward), and `batch_norm2d`
  (training statistics, running-stat update, fused backward).

The graph is built on a tensor type with the reference Tensor's protocol
(`gpu_buf`, `shape`, `requires_grad`, `grad`, `_ctx`, `_accumulate_grad`,
`from_gpu`, `sync`).  By default that is `directcompute_torch_b200.tensor.
DeviceTensor`; `bind(nn_engine)` makes the ops build on the reference's own
`nn_engine.Tensor` instead (its module loaded over this library as
`engine.dll`), so one tape holds both the reference's Functions and these ops.

There is no CPU fallback: the ops need libdct_cuda.so and a CUDA device.
"""
from __future__ import annotations

import builtins
import ctypes
import struct

import numpy as np

from . import load_library
from ._abi import BINARY, REDUCE, UNARY, check
from .tensor import DeviceTensor, Node

__all__ = ["add", "sub", "mul", "div", "maximum", "minimum", "exp", "log_abs1p", "tanh", "sigmoid", "neg",
           "abs", "sum", "mean", "max", "min", "argmax", "argmin", "sum_to_shape", "broadcast_to",
           "softmax_cross_entropy", "bias_relu", "batch_norm2d", "tensor", "to_numpy", "bind"]

lib = load_library()
Tensor = DeviceTensor


def bind(module=None):
    """Build the ops' graphs on `module.Tensor` (e.g. the reference's `nn_engine`,
    loaded over this library); `bind()` returns to DeviceTensor.  Returns the
    tensor type now in use."""
    global Tensor
    if module is None:
        Tensor = DeviceTensor
        return Tensor
    t = getattr(module, "Tensor", None)
    need = ("from_gpu", "sync", "_accumulate_grad", "backward")
    if t is None or not all(hasattr(t, a) for a in need):
        raise TypeError(f"bind: {module!r} has no Tensor type with {', '.join(need)}")
    Tensor = t
    _scalars.clear()
    return Tensor


def _shape_arr(shape):
    shape = tuple(int(d) for d in shape)
    return (ctypes.c_int64 * builtins.max(1, len(shape)))(*shape), len(shape)


def _size(shape):
    n = 1
    for d in shape:
        n *= int(d)
    return n


def _buf(n):
    h = lib.dct_create_buffer(builtins.max(1, int(n)))
    if not h:
        raise MemoryError("libdct_cuda: " + (lib.dct_last_error() or b"").decode())
    return h


_scalars = {}


def _wrap(h, shape, ctx=None, requires_grad=False):
    t = Tensor.from_gpu(h, tuple(shape), requires_grad=requires_grad)
    t._ctx = ctx
    return t


def _scalar(v: float):
    """A cached one-element device buffer holding float32(v)."""
    key = np.float32(v).tobytes()
    t = _scalars.get(key)
    if t is None:
        t = Tensor(np.array([v], np.float32), track=False)
        _scalars[key] = t
    return t


def tensor(data, requires_grad=False) -> Tensor:
    return Tensor(np.asarray(data, dtype=np.float32), requires_grad=requires_grad)


def to_numpy(t: Tensor) -> np.ndarray:
    return np.array(t.sync(), copy=True).reshape(t.shape)


# ---------------------------------------------------------------------------
# raw launches (no tape)
# ---------------------------------------------------------------------------
def _binary_raw(op: str, a_h, a_shape, b_h, b_shape):
    out_shape = tuple(np.broadcast_shapes(tuple(a_shape), tuple(b_shape)))
    h = _buf(_size(out_shape))
    A, na = _shape_arr(a_shape)
    B, nb = _shape_arr(b_shape)
    check(lib, lib.dct_binary(BINARY[op], a_h, A, na, b_h, B, nb, h), f"dct_binary({op})")
    return h, out_shape


def _unary_raw(op: str, x_h, n):
    h = _buf(n)
    check(lib, lib.dct_unary(UNARY[op], x_h, h, n, 0.0), f"dct_unary({op})")
    return h


def _sum_to_shape_raw(g_h, g_shape, t_shape):
    g_shape, t_shape = tuple(g_shape), tuple(t_shape)
    if g_shape == t_shape:
        lib.AddRefBuffer(g_h)
        return g_h
    h = _buf(_size(t_shape))
    G, ng = _shape_arr(g_shape)
    T, nt = _shape_arr(t_shape)
    check(lib, lib.dct_sum_to_shape(g_h, G, ng, T, nt, h), "dct_sum_to_shape")
    return h


def _broadcast_raw(x_h, x_shape, out_shape):
    x_shape, out_shape = tuple(x_shape), tuple(out_shape)
    if x_shape == out_shape:
        lib.AddRefBuffer(x_h)
        return x_h
    h = _buf(_size(out_shape))
    X, nx = _shape_arr(x_shape)
    O, no = _shape_arr(out_shape)
    check(lib, lib.dct_broadcast_to(x_h, X, nx, O, no, h), "dct_broadcast_to")
    return h


def _release(*hs):
    for h in hs:
        if h:
            lib.ReleaseBuffer(h)


def sum_to_shape(g: Tensor, shape) -> Tensor:
    """g summed over the dims where `shape` (right-aligned) broadcasts: the broadcast gradient."""
    return _wrap(_sum_to_shape_raw(g.gpu_buf, g.shape, shape), shape)


def broadcast_to(x: Tensor, shape) -> Tensor:
    return _wrap(_broadcast_raw(x.gpu_buf, x.shape, shape), shape)


# ---------------------------------------------------------------------------
# broadcast binary ops
# ---------------------------------------------------------------------------
class BinaryFunc(Node):
    def __init__(self, op):
        super().__init__()
        self.op = op

    def forward(self, a: Tensor, b: Tensor) -> Tensor:
        self.inputs = (a, b)
        h, shape = _binary_raw(self.op, a.gpu_buf, a.shape, b.gpu_buf, b.shape)
        out = _wrap(h, shape, self, a.requires_grad or b.requires_grad)
        if self.op == "div":
            self.out = out
        return out

    def _give(self, t: Tensor, full_h, full_shape, negate=False, fresh=False):
        """Hand t its share of the gradient.  A same-shape gradient aliases
        `full_h` (as the reference's AddFunc does) unless `fresh` asks for a
        private copy: two inputs must never share one gradient buffer, since
        a later accumulation into one would change the other."""
        if negate:
            h0 = _sum_to_shape_raw(full_h, full_shape, t.shape)
            h = _unary_raw("neg", h0, t.size)
            _release(h0)
        elif fresh and tuple(full_shape) == tuple(t.shape):
            h, _ = _binary_raw("copy", full_h, full_shape, full_h, full_shape)
        else:
            h = _sum_to_shape_raw(full_h, full_shape, t.shape)
        t._accumulate_grad(_wrap(h, t.shape))

    def backward(self, g: Tensor):
        a, b = self.inputs
        op, gs = self.op, g.shape
        if op in ("add", "sub"):
            if a.requires_grad:
                self._give(a, g.gpu_buf, gs)
            if b.requires_grad:
                self._give(b, g.gpu_buf, gs, negate=(op == "sub"), fresh=a.requires_grad)
        elif op == "mul":
            if a.requires_grad:
                h, _ = _binary_raw("mul", g.gpu_buf, gs, b.gpu_buf, b.shape)
                self._give(a, h, gs)
                _release(h)
            if b.requires_grad:
                h, _ = _binary_raw("mul", g.gpu_buf, gs, a.gpu_buf, a.shape)
                self._give(b, h, gs)
                _release(h)
        elif op == "div":
            q, _ = _binary_raw("div", g.gpu_buf, gs, b.gpu_buf, b.shape)           # g / b
            if a.requires_grad:
                self._give(a, q, gs)
            if b.requires_grad:                                                    # -(g / b) * (a / b)
                t, _ = _binary_raw("mul", q, gs, self.out.gpu_buf, self.out.shape)
                self._give(b, t, gs, negate=True)
                _release(t)
            _release(q)
        else:                                                                      # maximum / minimum
            pick = "pick_max" if op == "maximum" else "pick_min"
            m, _ = _binary_raw(pick, a.gpu_buf, a.shape, b.gpu_buf, b.shape)
            ga, _ = _binary_raw("mul", g.gpu_buf, gs, m, gs)                       # g where a wins
            if a.requires_grad:
                self._give(a, ga, gs)
            if b.requires_grad:
                gb, _ = _binary_raw("sub", g.gpu_buf, gs, ga, gs)                  # g where b wins (exact)
                self._give(b, gb, gs)
                _release(gb)
            _release(m, ga)


def _as_tensor(x):
    if isinstance(x, Tensor):
        return x
    return _scalar(float(x)) if np.ndim(x) == 0 else tensor(x)


def add(a, b): return BinaryFunc("add").forward(_as_tensor(a), _as_tensor(b))
def sub(a, b): return BinaryFunc("sub").forward(_as_tensor(a), _as_tensor(b))
def mul(a, b): return BinaryFunc("mul").forward(_as_tensor(a), _as_tensor(b))
def div(a, b): return BinaryFunc("div").forward(_as_tensor(a), _as_tensor(b))
def maximum(a, b): return BinaryFunc("maximum").forward(_as_tensor(a), _as_tensor(b))
def minimum(a, b): return BinaryFunc("minimum").forward(_as_tensor(a), _as_tensor(b))


# ---------------------------------------------------------------------------
# unary ops
# ---------------------------------------------------------------------------
class UnaryFunc(Node):
    # op -> (backward kernel, what it takes besides g: "y" the output or "x" the input)
    GRADS = {"exp": ("exp_grad", "y"), "tanh": ("tanh_grad", "y"), "sigmoid": ("sigmoid_grad", "y"),
             "log_abs1p": ("log_abs1p_grad", "x"), "neg": (None, None), "abs": (None, "x")}

    def __init__(self, op):
        super().__init__()
        self.op = op

    def forward(self, x: Tensor) -> Tensor:
        self.inputs = (x,)
        out = _wrap(_unary_raw(self.op, x.gpu_buf, x.size), x.shape, self, x.requires_grad)
        self.out = out
        return out

    def backward(self, g: Tensor):
        x = self.inputs[0]
        if not x.requires_grad:
            return
        kern, saved = self.GRADS[self.op]
        if self.op == "neg":
            h = _unary_raw("neg", g.gpu_buf, x.size)
        elif self.op == "abs":                                       # g * sign(x), sign(0) = 0
            zero = _scalar(0.0)
            p, _ = _binary_raw("pick_max", x.gpu_buf, x.shape, zero.gpu_buf, ())
            m, _ = _binary_raw("pick_min", x.gpu_buf, x.shape, zero.gpu_buf, ())
            s, _ = _binary_raw("sub", p, x.shape, m, x.shape)
            h, _ = _binary_raw("mul", g.gpu_buf, x.shape, s, x.shape)
            _release(p, m, s)
        else:
            other = self.out if saved == "y" else x
            h, _ = _binary_raw(kern, g.gpu_buf, x.shape, other.gpu_buf, x.shape)
        x._accumulate_grad(_wrap(h, x.shape))


def exp(x): return UnaryFunc("exp").forward(x)
def log_abs1p(x): return UnaryFunc("log_abs1p").forward(x)
def tanh(x): return UnaryFunc("tanh").forward(x)
def sigmoid(x): return UnaryFunc("sigmoid").forward(x)
def neg(x): return UnaryFunc("neg").forward(x)
def abs(x): return UnaryFunc("abs").forward(x)   # noqa: A001  (NumPy's name)


# ---------------------------------------------------------------------------
# reductions
# ---------------------------------------------------------------------------
def _view3(shape, axis):
    """[outer, len, inner] view of `shape` for a reduction over `axis` (None = all)."""
    if axis is None:
        return 1, _size(shape), 1, ()
    nd = len(shape)
    ax = axis + nd if axis < 0 else axis
    if not 0 <= ax < nd:
        raise ValueError(f"axis {axis} out of range for {nd} dims")
    outer = _size(shape[:ax])
    inner = _size(shape[ax + 1:])
    return outer, int(shape[ax]), inner, tuple(shape[:ax]) + tuple(shape[ax + 1:])


class ReduceFunc(Node):
    def __init__(self, op, axis, keepdims):
        super().__init__()
        self.op, self.axis, self.keepdims = op, axis, keepdims

    def forward(self, x: Tensor) -> Tensor:
        self.inputs = (x,)
        outer, n, inner, out_shape = _view3(x.shape, self.axis)
        if n == 0 and self.op not in ("sum", "mean"):
            raise ValueError(f"{self.op} of an empty axis")
        h = _buf(outer * inner)
        if self.axis is None and self.op in ("sum", "mean", "max", "min"):
            check(lib, lib.dct_reduce_all(REDUCE[self.op], x.gpu_buf, n, h, None), f"dct_reduce_all({self.op})")
        else:
            check(lib, lib.dct_reduce(REDUCE[self.op], x.gpu_buf, outer, n, inner, h, None), f"dct_reduce({self.op})")
        if self.keepdims:
            out_shape = tuple(1 if (self.axis is None or i == (self.axis % len(x.shape))) else d
                              for i, d in enumerate(x.shape))
        self.n = n
        differentiable = self.op in ("sum", "mean")
        return _wrap(h, out_shape, self, x.requires_grad and differentiable)

    def backward(self, g: Tensor):
        x = self.inputs[0]
        if not x.requires_grad:
            return
        if self.axis is None:
            kshape = (1,) * len(x.shape)
        else:
            ax = self.axis % len(x.shape)
            kshape = tuple(1 if i == ax else d for i, d in enumerate(x.shape))
        h = _broadcast_raw(g.gpu_buf, kshape, x.shape)                     # g viewed with keepdims
        if self.op == "mean":
            s = _scalar(1.0 / self.n)
            h2, _ = _binary_raw("mul", h, x.shape, s.gpu_buf, ())
            _release(h)
            h = h2
        x._accumulate_grad(_wrap(h, x.shape))


def sum(x, axis=None, keepdims=False): return ReduceFunc("sum", axis, keepdims).forward(x)    # noqa: A001
def mean(x, axis=None, keepdims=False): return ReduceFunc("mean", axis, keepdims).forward(x)
def max(x, axis=None, keepdims=False): return ReduceFunc("max", axis, keepdims).forward(x)    # noqa: A001
def min(x, axis=None, keepdims=False): return ReduceFunc("min", axis, keepdims).forward(x)    # noqa: A001


def _arg(op, x, axis):
    outer, n, inner, out_shape = _view3(x.shape, axis)
    if n == 0:
        raise ValueError(f"{op} of an empty axis")
    h = _buf(outer * inner)
    try:
        check(lib, lib.dct_reduce(REDUCE[op], x.gpu_buf, outer, n, inner, h, None), f"dct_reduce({op})")
        out = np.empty(outer * inner, np.float32)
        lib.ReadBuffer(h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    finally:
        _release(h)
    idx = out.view(np.int32).astype(np.int64)
    return idx.reshape(out_shape) if out_shape else int(idx[0])


def argmax(x, axis=None):
    """Index of the first maximum (NaN counts as the maximum), as NumPy int64."""
    return _arg("argmax", x, axis)


def argmin(x, axis=None):
    return _arg("argmin", x, axis)


# ---------------------------------------------------------------------------
# fused softmax + cross-entropy
# ---------------------------------------------------------------------------
class SoftmaxCrossEntropyFunc(Node):
    """Mean cross-entropy of row softmax; one kernel writes probs, the loss and dlogits."""

    def forward(self, logits: Tensor, labels: Tensor, want_probs=False):
        self.inputs = (logits, labels)
        B, K = logits.shape
        self.dlog = _buf(B * K)
        ph = _buf(B * K) if want_probs else None
        lh = _buf(1)
        check(lib, lib.dct_softmax_ce(logits.gpu_buf, labels.gpu_buf, 0, B, K, ph, self.dlog, lh, None,
                                      float(B), float(B)), "dct_softmax_ce")
        self.probs = _wrap(ph, (B, K)) if want_probs else None
        return _wrap(lh, (1,), self, logits.requires_grad)

    def backward(self, g: Tensor):
        x = self.inputs[0]
        if x.requires_grad:
            h, _ = _binary_raw("mul", self.dlog, x.shape, g.gpu_buf, (1,))
            x._accumulate_grad(_wrap(h, x.shape))

    def __del__(self):
        if getattr(self, "dlog", None):
            lib.ReleaseBuffer(self.dlog)
            self.dlog = None


def softmax_cross_entropy(logits: Tensor, labels: Tensor, return_probs=False):
    """Mean CE over rows (labels: float class ids, the reference's layout)."""
    f = SoftmaxCrossEntropyFunc()
    loss = f.forward(logits, labels, want_probs=return_probs)
    return (loss, f.probs) if return_probs else loss


# ---------------------------------------------------------------------------
# bias + ReLU with the fused backward, BatchNorm2d
# ---------------------------------------------------------------------------
def _run_shader(name: str, srvs, uavs, groups, words):
    """One reference dispatch by shader name with its cbuffer words; raises on a library error."""
    lib.CompileShader(name.encode(), "")
    lib.dct_clear_error()
    sv = (ctypes.c_void_p * builtins.max(1, len(srvs)))(*srvs)
    uv = (ctypes.c_void_p * builtins.max(1, len(uavs)))(*uavs)
    th = (ctypes.c_uint * 3)(*groups)
    cb = (ctypes.c_uint * builtins.max(1, len(words)))(*words)
    lib.RunShader(name.encode(), sv, len(srvs), uv, len(uavs), th, ctypes.cast(cb, ctypes.c_void_p), 4 * len(words))
    check(lib, lib.dct_error_code(), name)


def _f2u(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", float(v)))[0]


class BiasReLUFunc(Node):
    """y = max(0, x + b) over rows (nn_bias_relu.hlsl:8-12); the backward writes dx and db in
    one pass over the upstream gradient and y (dct_bias_relu_backward)."""

    def forward(self, x, b):
        self.inputs = (x, b)
        M, N = x.size // b.size, b.size
        if M * N != x.size or x.shape[-1] != N:
            raise ValueError(f"bias_relu: bias of {b.size} does not match the rows of {x.shape}")
        h = _buf(x.size)
        _run_shader("bias_relu", [x.gpu_buf, b.gpu_buf], [h], ((x.size + 255) // 256, 1, 1), [M, N])
        self.M, self.N = M, N
        self.out = _wrap(h, x.shape, self, x.requires_grad or b.requires_grad)
        return self.out

    def backward(self, g):
        x, b = self.inputs
        dx, db = _buf(x.size), _buf(b.size)
        check(lib, lib.dct_bias_relu_backward(g.gpu_buf, self.out.gpu_buf, dx, db, self.M, self.N),
              "dct_bias_relu_backward")
        if x.requires_grad:
            x._accumulate_grad(_wrap(dx, x.shape))
        else:
            _release(dx)
        if b.requires_grad:
            b._accumulate_grad(_wrap(db, b.shape))
        else:
            _release(db)


def bias_relu(x, b):
    """max(0, x + b) with b broadcast over the rows of x."""
    return BiasReLUFunc().forward(x, b)


class BatchNorm2dFunc(Node):
    """Training-mode BatchNorm over NCHW: batch statistics in float64, the running
    statistics updated with momentum and the unbiased variance, then the apply
    (nn_batchnorm_mean_var.hlsl, nn_batchnorm_forward.hlsl); the backward gives
    dx, dgamma and dbeta (nn_batchnorm_backward_reduce.hlsl,
    nn_batchnorm_backward_dx.hlsl) from two passes over x and dy."""

    def forward(self, x, gamma, beta, running_mean, running_var, momentum=0.1, eps=1e-5):
        if len(x.shape) != 4:
            raise ValueError("batch_norm2d: x must be NCHW")
        N, C, H, W = x.shape
        self.inputs = (x, gamma, beta)
        self.dims = (N, C, H * W)
        self.eps = float(eps)
        self.mean, self.var = _buf(C), _buf(C)
        h = _buf(x.size)
        check(lib, lib.dct_batchnorm_forward_train(x.gpu_buf, gamma.gpu_buf, beta.gpu_buf, running_mean.gpu_buf,
                                                   running_var.gpu_buf, self.mean, self.var, h, N, C, H * W,
                                                   float(eps), float(momentum)), "dct_batchnorm_forward_train")
        return _wrap(h, x.shape, self, x.requires_grad or gamma.requires_grad or beta.requires_grad)

    def backward(self, g):
        x, gamma, beta = self.inputs
        N, C, S = self.dims
        dx, dg, db = _buf(x.size), _buf(C), _buf(C)
        check(lib, lib.dct_batchnorm_backward(x.gpu_buf, g.gpu_buf, self.mean, self.var, gamma.gpu_buf, dg, db, dx,
                                              N, C, S, self.eps), "dct_batchnorm_backward")
        for t, h in ((x, dx), (gamma, dg), (beta, db)):
            if t.requires_grad:
                t._accumulate_grad(_wrap(h, t.shape))
            else:
                _release(h)

    def __del__(self):
        for k in ("mean", "var"):
            h = getattr(self, k, None)
            if h:
                try:
                    lib.ReleaseBuffer(h)
                except Exception:
                    pass
                setattr(self, k, None)


def batch_norm2d(x, gamma, beta, running_mean, running_var, training=True, momentum=0.1, eps=1e-5):
    """BatchNorm over NCHW.  Training: batch statistics (the running ones updated in
    place), differentiable in x, gamma and beta.  Evaluation: the running statistics,
    no gradient (the reference's eval path, nn_engine.py:1794-1868)."""
    if training:
        return BatchNorm2dFunc().forward(x, gamma, beta, running_mean, running_var, momentum, eps)
    N, C, H, W = x.shape
    h = _buf(x.size)
    _run_shader("batchnorm_forward", [x.gpu_buf, running_mean.gpu_buf, running_var.gpu_buf, gamma.gpu_buf,
                                      beta.gpu_buf], [h], ((x.size + 255) // 256, 1, 1), [N, C, H * W, _f2u(eps)])
    return _wrap(h, x.shape)
