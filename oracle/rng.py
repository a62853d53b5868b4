"""Host restatement of the library's synthetic-data generator -- TEST INFRASTRUCTURE ONLY.

`dct_fill_random` (directcompute_torch_b200/csrc/k_rng.cu) fills a buffer with
Philox4x32-10, the counter-based generator of Salmon, Moraes, Dror and Shaw,
"Parallel random numbers: as easy as 1, 2, 3" (SC'11).  The reference has no
generator of its own on this path (its inputs come from NumPy); this one exists
so that every rank can fill its own rows of the large benchmark inputs on the
device.  This module restates it on the host from the paper's definition:

* one round maps the counter (c0, c1, c2, c3) under key (k0, k1) to
  (hi(M1*c2) ^ c1 ^ k0, lo(M1*c2), hi(M0*c0) ^ c3 ^ k1, lo(M0*c0)) with the
  published multipliers M0 = 0xD2511F53, M1 = 0xCD9E8D57; the key is bumped by
  the Weyl constants (0x9E3779B9, 0xBB67AE85) between rounds; ten rounds;
* element i of a fill takes word i % 4 of the block for counter
  (i // 4 as two 32-bit words, offset as two 32-bit words) under key
  (seed low word, seed high word);
* uniform [a, b): u = (word >> 8) * 2^-24, then fl(fl(u * fl(b - a)) + a) in
  float32 -- every step is a correctly rounded float32 operation, so the host
  stream equals the device stream bit for bit;
* normal(mean a, std b): Box-Muller on the block's word pairs
  (u1 = ((w >> 8) + 1) * 2^-24 in (0, 1], u2 = (w' >> 8) * 2^-24), giving
  a + b * r * cos(2 pi u2) and a + b * r * sin(2 pi u2), r = sqrt(-2 ln u1).
  The device evaluates ln, sin and cos with CUDA's float32 functions, so the
  host returns the float64 value and tests hold the device within a stated
  error bound (`normal_error_bound`) instead of bit equality.

`KAT` holds the known-answer vectors that Random123 (the paper's reference
implementation) publishes for philox4x32 with 10 rounds.
"""
from __future__ import annotations

import numpy as np

M0 = np.uint64(0xD2511F53)
M1 = np.uint64(0xCD9E8D57)
W0 = 0x9E3779B9
W1 = 0xBB67AE85
MASK = np.uint64(0xFFFFFFFF)
TWO_M24 = 5.9604644775390625e-08          # 2^-24

#: (counter, key, output) triples published with Random123 for philox4x32-10
KAT = (
    ((0x00000000, 0x00000000, 0x00000000, 0x00000000), (0x00000000, 0x00000000),
     (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF), (0xFFFFFFFF, 0xFFFFFFFF),
     (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
)


def philox4x32_10(c0, c1, c2, c3, k0: int, k1: int):
    """Ten Philox4x32 rounds over arrays of counters (uint32-valued); returns four uint32 arrays."""
    c0, c1, c2, c3 = (np.asarray(v, dtype=np.uint64) & MASK for v in (c0, c1, c2, c3))
    k0 &= 0xFFFFFFFF
    k1 &= 0xFFFFFFFF
    for _ in range(10):
        p0 = M0 * c0                          # < 2^64: exact in uint64
        p1 = M1 * c2
        hi0, lo0 = p0 >> np.uint64(32), p0 & MASK
        hi1, lo1 = p1 >> np.uint64(32), p1 & MASK
        c0, c1, c2, c3 = hi1 ^ c1 ^ np.uint64(k0), lo1, hi0 ^ c3 ^ np.uint64(k1), lo0
        k0 = (k0 + W0) & 0xFFFFFFFF
        k1 = (k1 + W1) & 0xFFFFFFFF
    return tuple(v.astype(np.uint32) for v in (c0, c1, c2, c3))


def words(seed: int, offset: int, start: int, count: int) -> np.ndarray:
    """The 32-bit word that element i of a fill uses, for i in [start, start + count)."""
    if count <= 0:
        return np.zeros(0, np.uint32)
    g0, g1 = start // 4, (start + count - 1) // 4 + 1
    g = np.arange(g0, g1, dtype=np.uint64)
    out = philox4x32_10(g & MASK, g >> np.uint64(32), np.full_like(g, offset & 0xFFFFFFFF),
                        np.full_like(g, (offset >> 32) & 0xFFFFFFFF), seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF)
    w = np.stack(out, axis=1).ravel()
    lo = start - 4 * g0
    return w[lo:lo + count]


def uniform(seed: int, offset: int, start: int, count: int, a: float, b: float) -> np.ndarray:
    """Elements [start, start + count) of `dct_fill_random(.., seed, offset, dist=0, a, b)`, bit-exact."""
    w = words(seed, offset, start, count)
    u = ((w >> np.uint32(8)).astype(np.float32) * np.float32(TWO_M24)).astype(np.float32)
    width = np.float32(np.float32(b) - np.float32(a))
    return ((u * width).astype(np.float32) + np.float32(a)).astype(np.float32)


def normal_f64(seed: int, offset: int, start: int, count: int, mean: float, std: float) -> np.ndarray:
    """Elements [start, start + count) of a normal fill, evaluated in float64 from the same uniforms."""
    g0 = start // 4
    g1 = (start + count + 3) // 4                  # whole blocks: a pair's second word may lie past the end
    w = words(seed, offset, 4 * g0, 4 * (g1 - g0)).astype(np.uint64).reshape(-1, 2, 2)   # [block][pair][(a, b)]
    u1 = ((w[:, :, 0] >> np.uint64(8)) + np.uint64(1)).astype(np.float64) * TWO_M24
    u2 = (w[:, :, 1] >> np.uint64(8)).astype(np.float64) * TWO_M24
    r = np.sqrt(-2.0 * np.log(u1))
    out = np.empty((w.shape[0], 2, 2), np.float64)
    out[:, :, 0] = float(np.float32(mean)) + float(np.float32(std)) * (r * np.cos(2.0 * np.pi * u2))
    out[:, :, 1] = float(np.float32(mean)) + float(np.float32(std)) * (r * np.sin(2.0 * np.pi * u2))
    flat = out.ravel()
    lo = start - 4 * g0
    return flat[lo:lo + count]


def normal_error_bound(ref64: np.ndarray, mean: float, std: float) -> np.ndarray:
    """Allowed |device - float64| for a normal fill: 8 float32 ulps of |std * r| + |mean| (and one of the value).

    The device forms r from CUDA's logf (at most 1 ulp) and a correctly rounded
    sqrtf, the angle from sincospif (at most 1 ulp each), then one fused
    multiply-add with the mean; the bound covers those roundings with margin.
    """
    scale = np.abs(ref64 - float(np.float32(mean))) + abs(float(np.float32(mean)))
    return 8.0 * scale * 2.0 ** -24 + np.spacing(np.abs(ref64).astype(np.float32)).astype(np.float64)
