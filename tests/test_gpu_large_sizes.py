"""Operands past 2^32 elements, checked through exact properties on the device.

One buffer of 2^32 + 4099 fp32 (17 GB) exercises the library's 64-bit element
indexing:
- zeroed, then `exp` in place, it must read 1.0 everywhere;
- three values are then scattered past index 2^32, one of them the last element;
- the full sum and max over all of it, and axis sums over two views whose products
  exceed 2^32, must equal values computed here from the layout alone.

The sums are exact in float64 (integers and halves below 2^53), and each float32
output is that sum rounded once. No 17 GB array crosses PCIe: the checks read
back scalars and short rows. An arg reduction over an axis of 2^31 or more is
refused (the indices are int32), and so is a `dct_reduce` extent of 2^32 or more.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N = (1 << 32) + 4099


def test_past_two_to_the_32(dev):
    lib = dev.lib
    h = lib.dct_create_buffer(N)
    assert h, dev.error()
    try:
        assert lib.dct_buffer_count(h) == N
        lib.ClearBuffer(h)
        dev.unary("exp", h, h, N)                                # exp(0) = 1 everywhere, in place
        idx = np.array([(1 << 32) + 7, (1 << 32) + 4096, N - 1], np.int64)
        val = np.array([5.0, -2.0, 2.5], np.float32)
        rc = lib.dct_scatter(h, idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                             val.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), len(idx))
        assert rc == 0, dev.error()
        delta = {int(i): float(v) - 1.0 for i, v in zip(idx, val)}
        out = dev.empty(4096)
        assert dev.reduce_all("sum", h, N, out) == N + sum(delta.values())
        assert dev.reduce_all("max", h, N, out) == 5.0
        assert dev.reduce_all("min", h, N, out) == -2.0
        # axis -1 over [2, L, 1]: 2L = 2^32 + 4098 elements
        L = (N - 1) // 2
        dev.reduce("sum", h, 2, L, 1, out)
        want = np.full(2, float(L))
        for i, dv in delta.items():
            if i < 2 * L:
                want[i // L] += dv
        np.testing.assert_array_equal(dev.read(out)[:2], want.astype(np.float32))   # float64 sum, rounded once
        # axis 0 over [1, R, 4096]: R * 4096 = 2^32 + 4096 elements
        R = N // 4096
        dev.reduce("sum", h, 1, R, 4096, out)
        want = np.full(4096, float(R))
        for i, dv in delta.items():
            if i < R * 4096:
                want[i % 4096] += dv
        np.testing.assert_array_equal(dev.read(out), want.astype(np.float32))
        # arg reductions keep int32 indices: an axis of 2^31 or more is refused
        with pytest.raises(RuntimeError, match="ARG"):
            dev.reduce("argmax", h, 2, L, 1, out)
        with pytest.raises(RuntimeError, match="ARG"):
            dev.reduce("sum", h, 1, N, 1, out)                   # an extent of 2^32 or more
        dev.clear_error()
        dev.free(out)
    finally:
        lib.ReleaseBuffer(h)
        lib.DrainPool()
