"""Thin test helper over libdct_cuda.so's C-ABI (handles <-> NumPy arrays).

Everything goes through the exported entry points -- CreateBuffer/ReadBuffer,
RunShader with the reference's cbuffer words, and the dct_* extensions -- so
the GPU tests exercise exactly what a reference caller would.
"""
from __future__ import annotations

import ctypes
import struct

import numpy as np

from directcompute_torch_b200 import load_library
from directcompute_torch_b200._abi import BINARY, REDUCE, UNARY, check


def f2u(f: float) -> int:
    return struct.unpack("<I", struct.pack("<f", float(f)))[0]


class Dev:
    def __init__(self):
        self.lib = load_library()
        if not self.lib.InitEngine():
            raise RuntimeError("libdct_cuda InitEngine failed: " + self.lib.dct_last_error().decode())
        from tests.names import HOT_PATH_SHADERS
        for n in HOT_PATH_SHADERS:
            self.lib.CompileShader(n.encode(), "")
        self._srv = (ctypes.c_void_p * 16)()
        self._uav = (ctypes.c_void_p * 16)()
        self._thr = (ctypes.c_uint * 3)()

    # -- buffers -----------------------------------------------------------
    def buf(self, arr) -> int:
        a = np.ascontiguousarray(arr)
        if a.dtype not in (np.float32, np.int32, np.uint32):
            a = a.astype(np.float32)
        a = a.view(np.float32).ravel()
        h = self.lib.CreateBuffer(a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), a.size)
        assert h, self.lib.dct_last_error()
        return h

    def empty(self, n: int, fill=None) -> int:
        h = self.lib.dct_create_buffer(int(n))
        assert h, self.lib.dct_last_error()
        if fill is not None:
            a = np.full(n, fill, dtype=np.float32)
            self.lib.UpdateBuffer(h, a.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        else:
            self.lib.ClearBuffer(h)
        return h

    def read(self, h, dtype=np.float32) -> np.ndarray:
        n = int(self.lib.dct_buffer_count(h))
        out = np.empty(n, dtype=np.float32)
        self.lib.ReadBuffer(h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        return out.view(dtype)

    def free(self, *hs):
        for h in hs:
            self.lib.ReleaseBuffer(h)

    def sync(self):
        check(self.lib, self.lib.dct_synchronize(), "synchronize")

    def error(self):
        return self.lib.dct_error_code(), (self.lib.dct_last_error() or b"").decode()

    def clear_error(self):
        self.lib.dct_clear_error()

    # -- dispatch -------------------------------------------------------------
    def run(self, name, srvs, uavs, groups, words=(), cb_bytes=None):
        for i, h in enumerate(srvs):
            self._srv[i] = h
        for i, h in enumerate(uavs):
            self._uav[i] = h
        self._thr[0], self._thr[1], self._thr[2] = groups
        if cb_bytes is None:
            cb_bytes = struct.pack("<%dI" % len(words), *[int(w) & 0xFFFFFFFF for w in words]) if words else b""
        cb = ctypes.create_string_buffer(cb_bytes, max(1, len(cb_bytes)))
        self.lib.RunShader(name.encode(), self._srv, len(srvs), self._uav, len(uavs), self._thr,
                           ctypes.cast(cb, ctypes.c_void_p) if cb_bytes else None, len(cb_bytes))

    # -- extension ops --------------------------------------------------------------
    def unary(self, op, x, y, n, alpha=0.0):
        check(self.lib, self.lib.dct_unary(UNARY[op], x, y, n, alpha), "dct_unary")

    def binary(self, op, a, ashape, b, bshape, out):
        A = (ctypes.c_int64 * max(1, len(ashape)))(*ashape)
        B = (ctypes.c_int64 * max(1, len(bshape)))(*bshape)
        check(self.lib, self.lib.dct_binary(BINARY[op], a, A, len(ashape), b, B, len(bshape), out), "dct_binary")

    def reduce(self, op, x, outer, length, inner, out, idx=None):
        check(self.lib, self.lib.dct_reduce(REDUCE[op], x, outer, length, inner, out, idx), "dct_reduce")

    def reduce_all(self, op, x, n, out):
        v = ctypes.c_double(0.0)
        check(self.lib, self.lib.dct_reduce_all(REDUCE[op], x, n, out, ctypes.byref(v)), "dct_reduce_all")
        return v.value
