"""A device tensor over one libdct_cuda buffer handle, with reverse-mode autograd.

The NumPy-semantics ops (`directcompute_torch_b200.ops`) build their graph on a
tensor type; this module is the one they use unless `ops.bind()` hands them the
reference's own `nn_engine` module instead.  To work with either, both follow
the same small protocol, the one the reference's Tensor exposes
(nn_engine.py:517-610):

* ``gpu_buf``       the library handle (a refcounted buffer of float32);
* ``shape`` / ``size``;
* ``requires_grad`` / ``grad`` (a tensor, or None);
* ``_ctx``          the node that produced the tensor: an object with an
  ``inputs`` tuple and ``backward(grad)``, which hands each input its share
  through ``input._accumulate_grad(g)``;
* ``from_gpu(handle, shape, requires_grad=False, track=True)`` wraps a handle
  whose one reference the new tensor takes over; ``sync()`` reads the values.

The tensor releases its reference of the handle when it is collected.
Gradients that meet at one tensor are added into a fresh buffer (never in
place), so a gradient buffer shared with another tensor is never modified.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import load_library
from ._abi import BINARY, check

__all__ = ["DeviceTensor", "Node"]


class Node:
    """Base of a graph node: the inputs it was applied to and its backward."""

    def __init__(self, *inputs):
        self.inputs = inputs

    def backward(self, grad):                      # pragma: no cover - every op overrides it
        raise NotImplementedError


def _new_handle(n: int):
    lib = load_library()
    h = lib.dct_create_buffer(max(1, int(n)))
    if not h:
        raise MemoryError("libdct_cuda: " + (lib.dct_last_error() or b"").decode())
    return h


class DeviceTensor:
    __slots__ = ("gpu_buf", "shape", "size", "requires_grad", "grad", "_ctx", "__weakref__")

    def __init__(self, data, requires_grad: bool = False, track: bool = True):
        lib = load_library()
        a = np.ascontiguousarray(data, dtype=np.float32)
        self.shape = tuple(a.shape)
        self.size = int(a.size)
        self.gpu_buf = _new_handle(self.size)
        if self.size:
            check(lib, lib.dct_copy_h2d(self.gpu_buf, a.ctypes.data_as(ctypes.c_void_p), 0, self.size), "upload")
            check(lib, lib.dct_synchronize(), "upload")
        self.requires_grad = bool(requires_grad)
        self.grad = None
        self._ctx = None

    @classmethod
    def from_gpu(cls, handle, shape, requires_grad: bool = False, track: bool = True) -> "DeviceTensor":
        t = object.__new__(cls)
        t.gpu_buf = handle
        t.shape = tuple(int(d) for d in shape)
        n = 1
        for d in t.shape:
            n *= d
        t.size = n
        t.requires_grad = bool(requires_grad)
        t.grad = None
        t._ctx = None
        return t

    def __del__(self):
        h = getattr(self, "gpu_buf", None)
        if h:
            try:
                load_library().ReleaseBuffer(h)
            except Exception:                      # interpreter shutdown
                pass
            self.gpu_buf = None

    def sync(self) -> np.ndarray:
        """The values, read back from the device (blocking)."""
        out = np.empty(self.shape, dtype=np.float32)
        if self.size:
            load_library().ReadBuffer(self.gpu_buf, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        return out

    numpy = sync

    def _accumulate_grad(self, g) -> None:
        if self.grad is None:
            self.grad = g
            return
        lib = load_library()
        h = _new_handle(self.size)
        shp = (ctypes.c_int64 * max(1, len(self.shape)))(*self.shape)
        check(lib, lib.dct_binary(BINARY["add"], self.grad.gpu_buf, shp, len(self.shape), g.gpu_buf, shp,
                                  len(self.shape), h), "gradient accumulation")
        self.grad = DeviceTensor.from_gpu(h, self.shape)

    def backward(self, grad=None) -> None:
        """Reverse-mode sweep from this tensor: every node runs once, after all the
        nodes that consume its output (an explicit-stack depth-first post-order)."""
        if grad is None:
            grad = DeviceTensor(np.ones(self.shape, dtype=np.float32))
        self.grad = grad
        order, seen = [], set()
        stack = [(self, False)]
        while stack:
            t, expanded = stack.pop()
            if expanded:
                order.append(t)
                continue
            if id(t) in seen:
                continue
            seen.add(id(t))
            stack.append((t, True))
            ctx = t._ctx
            if ctx is not None:
                for i in getattr(ctx, "inputs", ()):
                    if getattr(i, "requires_grad", False) and id(i) not in seen:
                        stack.append((i, False))
        for t in reversed(order):
            if t._ctx is not None and t.grad is not None:
                t._ctx.backward(t.grad)

    def __repr__(self):
        return f"DeviceTensor(shape={self.shape}, requires_grad={self.requires_grad})"
