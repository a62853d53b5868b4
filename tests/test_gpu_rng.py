"""dct_fill_random against the host Philox4x32-10 restatement (oracle/rng.py).

Uniform fills are bit-exact.  Normal fills use CUDA's float32 logf / sincospif,
so they are held to oracle.rng.normal_error_bound against the float64 value of
the same uniforms.  Every fill the benchmark makes (seed, offset, distribution)
is checked on a prefix and on an interior slice; element i depends only on
(seed, offset, i), so a shorter buffer holds the same prefix as the full one.
"""
import ctypes

import numpy as np
import pytest

from oracle import rng

pytestmark = pytest.mark.gpu

# (what, seed, offset, dist, a, b) for the bench's fills of each config
FILLS = [
    ("C1 X", 0, 0, 1, 0.0, 1.0), ("C1 b", 0, 1, 0, -0.1, 0.1),
    ("C2 A", 1, 0, 1, 0.0, 1.0), ("C2 B", 1, 1, 0, 0.5, 2.0), ("C2 C", 1, 2, 1, 0.0, 1.0),
    ("C2 D", 1, 3, 1, 0.0, 1.0),
    ("C3 R", 2, 0, 1, 0.0, 1.0), ("C3 V", 2, 7, 0, -1.0, 1.0),
    ("C4 logits", 3, 0, 1, 0.0, 3.0),
    ("C5a p", 4, 0, 1, 0.0, 0.02), ("C5a g", 4, 1, 1, 0.0, 1e-3),
    ("C5b x", 4, 10, 1, 0.5, 2.0), ("C5b dy", 4, 11, 1, 0.0, 1.0),
    ("rank 3 of C2 A", 3001, 0, 1, 0.0, 1.0), ("64-bit seed and offset", 0x1234_5678_9ABC, 1 << 40, 0, -3.0, 5.0),
]


@pytest.mark.parametrize("fill", FILLS, ids=[f[0] for f in FILLS])
def test_fill_matches_host_stream(dev, fill):
    _, seed, offset, dist, a, b = fill
    n = (1 << 20) + 3                       # ragged tail: the last block is partly used
    h = dev.empty(n)
    assert dev.lib.dct_fill_random(h, seed, offset, dist, a, b) == 0, dev.error()
    got = dev.read(h)
    for start, cnt in ((0, 1 << 16), (n - 4099, 4099)):
        sl = got[start:start + cnt]
        if dist == 0:
            want = rng.uniform(seed, offset, start, cnt, a, b)
            assert np.array_equal(sl.view(np.uint32), want.view(np.uint32))
        else:
            ref = rng.normal_f64(seed, offset, start, cnt, a, b)
            err = np.abs(sl.astype(np.float64) - ref)
            bound = rng.normal_error_bound(ref, a, b)
            assert (err <= bound).all(), (float((err / bound).max()), int((err / bound).argmax()))
    dev.free(h)


def test_offset_slices_of_a_copy(dev):
    """dct_copy_d2h with an element offset reads the same values as the host stream."""
    n = 3 << 20
    h = dev.empty(n)
    assert dev.lib.dct_fill_random(h, 9, 0, 0, 0.0, 1.0) == 0
    part = np.empty(1000, np.float32)
    assert dev.lib.dct_copy_d2h(h, part.ctypes.data_as(ctypes.c_void_p), n - 1000, 1000) == 0
    assert np.array_equal(part, rng.uniform(9, 0, n - 1000, 1000, 0.0, 1.0))
    dev.free(h)
