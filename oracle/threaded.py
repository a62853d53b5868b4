"""Multi-core timing of the NumPy oracle (the reported CPU baseline) -- test/bench infrastructure.

NumPy ufuncs release the GIL, so splitting the leading dimension over a thread
pool runs the reference's CPU arithmetic on every host core.  Only bench.py's
`cpu_baseline` / `--impl reference` legs call this.
"""
from __future__ import annotations

import concurrent.futures as cf
import time

import numpy as np

from . import newops as O

F32 = np.float32


def _chunks(n, k):
    step = (n + k - 1) // k
    return [(i, min(n, i + step)) for i in range(0, n, step)]


def c2_sample(threads: int, rows: int = 1024, reps: int = 3, seed: int = 1, min_seconds: float = 0.0,
              warmup: int = 1):
    """The 11 ops of BASELINE config C2 on a `rows`-row sample (same columns, same
    distributions): `warmup` untimed passes, then at least `reps` timed passes and
    at least `min_seconds` of them.  Returns (GB/s of algorithmic bytes over all
    timed passes, seconds per pass, text, timed passes)."""
    rng = np.random.default_rng(seed)
    cols = 8192
    A = rng.standard_normal((rows, cols), dtype=F32)
    B = (rng.random((1, cols), dtype=F32) * F32(1.5) + F32(0.5)).astype(F32)
    p = max(1, (64 * rows) // 8192)                 # outer-broadcast sample keeps the 64:512 ratio
    C = rng.standard_normal((p, 1, 4096), dtype=F32)
    D = rng.standard_normal((1, 512, 4096), dtype=F32)
    outA = np.empty_like(A)
    outO = np.empty((p, 512, 4096), dtype=F32)
    ufunc = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "div": np.divide, "maximum": np.maximum}
    pool = cf.ThreadPoolExecutor(max_workers=threads)
    rch = _chunks(rows, threads)
    pch = _chunks(p * 512, threads)
    C2 = C.reshape(p, 1, 4096)
    outO2 = outO.reshape(p * 512, 4096)

    def rowbcast(op):
        list(pool.map(lambda s: ufunc[op](A[s[0]:s[1]], B, out=outA[s[0]:s[1]]), rch))

    def outer(op):
        def part(s):
            for r in range(s[0], s[1]):
                ufunc[op](C2[r // 512, 0], D[0, r % 512], out=outO2[r])
        list(pool.map(part, pch))

    def unary(op):
        def part(s):
            outA[s[0]:s[1]] = O.unary_np32(op, A[s[0]:s[1]])
        list(pool.map(part, rch))

    plan = [(rowbcast, op, 4 * (2 * rows * cols + cols)) for op in ("add", "sub", "mul", "div", "maximum")]
    plan += [(outer, op, 4 * (p * 512 * 4096 + p * 4096 + 512 * 4096)) for op in ("mul", "add")]
    plan += [(unary, op, 4 * 2 * rows * cols) for op in ("exp", "log_abs1p", "tanh", "sigmoid")]
    total = sum(b for _, _, b in plan)
    with np.errstate(all="ignore"):
        for _ in range(max(0, warmup)):
            for fn, op, _ in plan:
                fn(op)
        passes = 0
        t0 = time.perf_counter()
        while passes < reps or time.perf_counter() - t0 < min_seconds:
            for fn, op, _ in plan:
                fn(op)
            passes += 1
        elapsed = time.perf_counter() - t0
    pool.shutdown()
    desc = (f"C2 sample: A[{rows},8192] (1/{8192 // rows} of the rows), C[{p},1,4096] x D[1,512,4096]; "
            f"11 ops; {passes} timed passes in {elapsed:.1f} s (mean), {threads} threads")
    return total * passes / elapsed / 1e9, elapsed / passes, desc, passes
