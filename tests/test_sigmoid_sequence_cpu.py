"""The device sigmoid's operation sequence, emulated exactly on the CPU.

`csrc/dct_math.cuh:sigmoid_tab` computes the sigmoid from Tang's table-driven
exponential and one remainder-corrected quotient.  This file restates that
sequence operation by operation in NumPy with correctly rounded float32
arithmetic:
- a multiply is exact in float64, then rounded once;
- an add or fused multiply-add goes through an error-free two-sum, then is rounded
  once via round-to-odd.

It then measures the error against float64 over a strided sweep of every binade
that matters, plus random arguments.  The hardware's approximate reciprocal is
not specified bit for bit, so every case also runs with it one ulp low and one
ulp high.  The bound asserted is the one the library documents: 1.5 ulp, with
the bar at 2 ulp.

The table of 2^(j/32 - 64) is parsed from the source and checked against
60-digit decimal arithmetic: hi is the float nearest the value and lo the float
nearest the rest.
"""
import os
import re
from decimal import Decimal, getcontext

import numpy as np
import pytest

F32, F64 = np.float32, np.float64
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "directcompute_torch_b200", "csrc", "dct_math.cuh")


def _table():
    src = open(SRC).read()
    body = src[src.index("kExp2Tab[32] = {"):]
    body = body[:body.index("};")]
    pairs = re.findall(r"\{\s*([^,{]+),\s*([^}]+)\}", body)

    def lit(t):
        t = t.strip().rstrip("f")
        return float.fromhex(t) if "x" in t else float(t)
    hi = np.array([lit(a) for a, _ in pairs], F32)
    lo = np.array([lit(b) for _, b in pairs], F32)
    return hi, lo


TH, TL = _table()


def _twosum(a, b):
    s = a + b
    bb = s - a
    return s, (a - (s - bb)) + (b - bb)


def _rn32(hi, lo):
    """Round the exact value hi + lo (hi = its float64 rounding) to float32 once."""
    odd = (hi.view(np.int64) & 1) == 1
    need = (lo != 0) & ~odd & np.isfinite(hi)
    hi = np.where(need, np.nextafter(hi, np.where(lo > 0, np.inf, -np.inf)), hi)
    return hi.astype(F32)


def _add(a, b):
    return _rn32(*_twosum(a.astype(F64), b.astype(F64)))


def _mul(a, b):
    return (a.astype(F64) * b.astype(F64)).astype(F32)


def _fma(a, b, c):
    return _rn32(*_twosum(a.astype(F64) * b.astype(F64), np.broadcast_to(c, a.shape).astype(F64)))


def _c(v, like):
    return np.full_like(like, F32(v))


def sigmoid_sequence(x, rcp_ulps=0):
    """sigmoid_tab, step for step (comments name the device statements)."""
    x = np.asarray(x, F32)
    with np.errstate(all="ignore"):
        a = np.abs(x)
        a = np.where(np.isnan(a), a, np.minimum(a, F32(104.0))).astype(F32)      # fmin_nanp(|x|, 104)
        magic = F32(12582912.0)
        kb = _fma(-a, _c(float.fromhex("0x1.715476p+5"), a), _c(magic, a))     # kb
        kf = _add(kb, -_c(magic, a))                                             # kf
        k = kb.view(np.int32) - magic.view(np.int32)                              # k
        r = _fma(-kf, _c(float.fromhex("0x1.62ep-6"), a), -a)
        r = _fma(-kf, _c(float.fromhex("0x1.0bfbe8p-20"), a), r)
        w = _fma(r, _c(float.fromhex("0x1.555556p-3"), a), _c(0.5, a))
        p = _fma(w, _mul(r, r), r)
        th, tl = TH[k & 31], TL[k & 31]
        ef = _add(th, _fma(th, p, tl))
        sc = (((k >> 5) + 191) << 23).astype(np.int32).view(F32)
        e = _mul(ef, sc)
        one = _c(1.0, a)
        s = _add(one, e)
        n = np.where(x < 0, e, one).astype(F32)
        rc = (1.0 / s.astype(F64)).astype(F32)                                   # rcp_approx(s), +- ulps
        for _ in range(abs(rcp_ulps)):
            rc = np.nextafter(rc, F32(np.inf) if rcp_ulps > 0 else F32(0))
        q0 = _mul(n, rc)
        rho = _fma(-q0, e, _add(n, -q0))
        return _fma(rho, rc, q0)


def _ulps(x, got):
    with np.errstate(all="ignore"):
        ex = 1.0 / (1.0 + np.exp(-x.astype(F64)))
    r32 = np.abs(ex.astype(F32))
    sp = np.spacing(r32).astype(F64)
    below = np.abs(ex) < r32.astype(F64)             # rounded up across a binade edge: the finer spacing
    sp = np.where(below, np.spacing(np.nextafter(r32, F32(0))).astype(F64), sp)
    sp = np.maximum(sp, 2.0 ** -149)                  # subnormal results: their spacing is the ulp
    return np.abs(got.astype(F64) - ex) / sp


def test_table_is_two_to_the_j_over_32_scaled():
    getcontext().prec = 60
    ln2 = Decimal(2).ln()
    assert TH.size == TL.size == 32
    for j in range(32):
        v = (Decimal(j) / 32 * ln2).exp() * Decimal(2) ** -64
        hi = F32(float(v))
        assert hi == TH[j], j
        rest = v - Decimal(float(hi))
        assert F32(float(rest)) == TL[j], j


def _sweep(stride):
    lo, hi = np.float32(2.0 ** -30).view(np.uint32), np.float32(110.0).view(np.uint32)
    xs = np.arange(int(lo) + 3, int(hi), stride, dtype=np.int64).astype(np.uint32).view(F32)
    r = np.random.default_rng(5)
    return np.concatenate([xs, -xs, r.uniform(-110, 110, 1 << 19).astype(F32),
                           r.uniform(-20, 20, 1 << 19).astype(F32),
                           np.array([0.0, -0.0, 104.0, -104.0, -87.33655, 20.0, -20.0, 1e-30, -1e-30], F32)])


@pytest.mark.parametrize("rcp_ulps", [-1, 0, 1])
def test_sequence_within_documented_bound(rcp_ulps):
    x = _sweep(4999)
    u = _ulps(x, sigmoid_sequence(x, rcp_ulps))
    assert u.max() <= 1.5, f"{u.max():.3f} ulp at x={x[u.argmax()]!r}"


def test_special_values():
    x = np.array([np.inf, -np.inf, np.nan, 0.0, -0.0, 200.0, -200.0], F32)
    y = sigmoid_sequence(x)
    assert y[0] == 1.0 and y[1] == 0.0 and np.isnan(y[2])
    assert y[3] == 0.5 and y[4] == 0.5 and y[5] == 1.0 and y[6] == 0.0
