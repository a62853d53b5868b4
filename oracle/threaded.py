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


def _timed(fn, reps: int, min_seconds: float, warmup: int = 1):
    """`warmup` untimed calls, then at least `reps` timed calls and at least `min_seconds`."""
    for _ in range(max(0, warmup)):
        fn()
    n = 0
    t0 = time.perf_counter()
    while n < reps or time.perf_counter() - t0 < min_seconds:
        fn()
        n += 1
    return (time.perf_counter() - t0) / n, n


def c1_sample(threads: int = 1, M: int = 256, N: int = 784, seed: int = 0, reps: int = 500,
              min_seconds: float = 1.0):
    """Config C1 whole, as NumPy runs it on the CPU (one thread: the arrays are 0.8 MB):
    Y = relu(X + b), sum(Y, axis=0), sum(Y), dX = relu_grad(ones, Y), db = sum(dX, axis=0),
    acc += db.  The vectorised forms are checked once against the oracle's formulas for
    nn_bias_relu.hlsl, nn_bias_grad.hlsl, nn_relu_grad.hlsl and nn_grad_accum.hlsl (same
    bits; the sums in float64), then timed.  `threads` is ignored.  Returns (GB/s over the
    chain's algorithmic bytes, seconds per step, text)."""
    from . import shaders as S
    rng = np.random.default_rng(seed)
    X = rng.standard_normal((M, N), dtype=F32)
    b = rng.uniform(-0.1, 0.1, N).astype(F32)
    ones = np.ones((M, N), F32)
    acc = np.zeros(N, F32)
    zero = F32(0.0)

    def chain(acc):
        Y = np.maximum(X + b, zero)
        s0 = Y.sum(axis=0, dtype=np.float64).astype(F32)
        tot = Y.sum(dtype=np.float64)
        dX = np.where(Y > 0, ones, zero)
        db = dX.sum(axis=0, dtype=np.float64).astype(F32)
        return Y, s0, tot, dX, db, acc + db

    Y, s0, _, dX, db, acc1 = chain(acc)
    assert np.array_equal(Y.ravel(), S.bias_relu(X.ravel(), b, M, N))
    assert np.array_equal(s0, S.bias_grad(Y.ravel(), M, N, N, 1))
    assert np.array_equal(dX.ravel(), S.relu_grad(ones.ravel(), Y.ravel(), M * N))
    assert np.array_equal(db, S.bias_grad(dX.ravel(), M, N, N, 1))
    assert np.array_equal(acc1, S.grad_accum(acc, db, N))

    def step():
        nonlocal acc
        acc = chain(acc)[-1]
    secs, n = _timed(step, reps, min_seconds)
    nbytes = 4 * (3 * M * N + 2 * N + 1) + 4 * (3 * M * N + N)
    desc = (f"C1 whole: X[{M},{N}] forward + backward chain (6 ops) per step, "
            f"{secs * 1e6:.0f} us per step; {n} steps, 1 thread")
    return nbytes / secs / 1e9, secs, desc


def c3_sample(threads: int, rows: int = 2048, cols: int = 4096, seed: int = 2, reps: int = 2,
              min_seconds: float = 2.0):
    """Config C3's eight axis reductions (sum / mean / max / argmax along axis -1 and
    axis 0) on a `rows`-row sample of R with the same outliers, each thread taking a
    block of rows (axis 0: per-block float64 column partials combined in block order).
    Returns (GB/s of algorithmic bytes, seconds per pass, text)."""
    rng = np.random.default_rng(seed)
    R = rng.standard_normal((rows, cols), dtype=F32)
    k = R.size // 1000
    idx = rng.choice(R.size, k, replace=False)
    R.flat[idx] = np.where(rng.integers(0, 2, k) == 1, 1e4, -1e4).astype(F32)
    pool = cf.ThreadPoolExecutor(max_workers=threads)
    rch = _chunks(rows, threads)

    def axis_last():
        def part(s):
            blk = R[s[0]:s[1]]
            sm = np.sum(blk, axis=1, dtype=np.float64)
            return sm.astype(F32), (sm / cols).astype(F32), blk.max(axis=1), blk.argmax(axis=1)
        list(pool.map(part, rch))

    def axis_first():
        def part(s):
            blk = R[s[0]:s[1]]
            return np.sum(blk, axis=0, dtype=np.float64), blk.max(axis=0), blk.argmax(axis=0) + s[0]
        parts = list(pool.map(part, rch))
        sm = sum(p[0] for p in parts)
        (sm / rows).astype(F32)
        mx = np.stack([p[1] for p in parts])
        win = mx.argmax(axis=0)                       # first block holding the maximum: first index
        np.stack([p[2] for p in parts])[win, np.arange(cols)]

    def step():
        axis_last()
        axis_first()
    secs, n = _timed(step, reps, min_seconds)
    pool.shutdown()
    nbytes = 4 * (4 * (rows * cols + rows) + 4 * (rows * cols + cols))
    desc = f"C3 sample: R[{rows},{cols}] (1/{16384 // rows} of the rows), 8 axis reductions; {n} passes, {threads} threads"
    return nbytes / secs / 1e9, secs, desc


def c4_sample(threads: int, rows: int = 8192, K: int = 1000, seed: int = 3, reps: int = 2, min_seconds: float = 2.0):
    """Config C4's fused softmax + cross-entropy forward and backward (probs, mean loss,
    dlogits) on a `rows`-row sample, float64 per row as the oracle computes it."""
    rng = np.random.default_rng(seed)
    X = (F32(3.0) * rng.standard_normal((rows, K), dtype=F32)).astype(F32)
    lab = rng.integers(0, K, rows).astype(np.int32)
    pool = cf.ThreadPoolExecutor(max_workers=threads)
    rch = _chunks(rows, threads)

    def step():
        def part(s):
            p, row_loss, _ = O.softmax_ce_rows_f64(X[s[0]:s[1]], lab[s[0]:s[1]])
            O.softmax_ce_dlogits(p, lab[s[0]:s[1]], rows)
            return float(row_loss.sum())
        sum(pool.map(part, rch)) / rows
    secs, n = _timed(step, reps, min_seconds)
    pool.shutdown()
    nbytes = 4 * (3 * rows * K + rows) + 4
    desc = f"C4 sample: logits[{rows},{K}] (1/{65536 // rows} of the rows), fused softmax+CE fwd+bwd; {n} passes, {threads} threads"
    return nbytes / secs / 1e9, secs, desc


def c5a_sample(threads: int, n: int = 30_000_000, seed: int = 4, reps: int = 2, min_seconds: float = 2.0):
    """Config C5a's Adam step (nn_adam.hlsl:18-34 restated) on an `n`-element subsample,
    each thread updating contiguous slices."""
    from . import shaders as S
    rng = np.random.default_rng(seed)
    w = (F32(0.02) * rng.standard_normal(n, dtype=F32)).astype(F32)
    g = (F32(1e-3) * rng.standard_normal(n, dtype=F32)).astype(F32)
    m = np.zeros(n, F32)
    v = np.zeros(n, F32)
    pool = cf.ThreadPoolExecutor(max_workers=threads)
    ch = _chunks(n, max(threads, n // (1 << 22)))
    t = [0]

    def step():
        t[0] += 1
        sz = S.adam_step_size(1e-3, 0.9, 0.999, t[0])

        def part(s):
            sl = slice(s[0], s[1])
            w[sl], m[sl], v[sl] = S.adam(w[sl], m[sl], v[sl], g[sl], s[1] - s[0], sz, 0.9, 0.999, 1e-8, 0.0, 1.0)
        list(pool.map(part, ch))
    secs, k = _timed(step, reps, min_seconds)
    pool.shutdown()
    desc = f"C5a sample: Adam on {n:.2e} elements (1/{1_500_000_000 // n} of 1.5e9); {k} steps, {threads} threads"
    return 28 * n / secs / 1e9, secs, desc


def c5b_sample(threads: int, N: int = 16, C: int = 256, S_: int = 56 * 56, seed: int = 4, reps: int = 1,
               min_seconds: float = 2.0):
    """Config C5b's BatchNorm training forward (statistics, then the apply) and backward
    (dgamma / dbeta, then dx) on an N-sample slice of the batch, each thread taking a
    block of samples (float64 channel partials combined in block order)."""
    from . import shaders as S
    rng = np.random.default_rng(seed)
    x = (F32(0.5) + F32(2.0) * rng.standard_normal(N * C * S_, dtype=F32)).astype(F32)
    dy = rng.standard_normal(N * C * S_, dtype=F32)
    gamma, beta = np.ones(C, F32), np.zeros(C, F32)
    pool = cf.ThreadPoolExecutor(max_workers=threads)
    nch = _chunks(N, threads)
    plane = C * S_
    eps = F32(1e-5)

    def step():
        def stats(s):
            X = x[s[0] * plane:s[1] * plane].reshape(-1, C, S_)
            return np.sum(X, axis=(0, 2), dtype=np.float64), np.sum(np.square(X, dtype=np.float64), axis=(0, 2))
        parts = list(pool.map(stats, nch))
        cnt = N * S_
        mean = sum(p[0] for p in parts) / cnt
        var = np.maximum(0.0, sum(p[1] for p in parts) / cnt - mean * mean)
        m32, v32 = mean.astype(F32), var.astype(F32)

        def fwd(s):
            sl = slice(s[0] * plane, s[1] * plane)
            return S.batchnorm_forward(x[sl], m32, v32, gamma, beta, s[1] - s[0], C, S_, eps)
        list(pool.map(fwd, nch))

        def red(s):
            sl = slice(s[0] * plane, s[1] * plane)
            X = x[sl].reshape(-1, C, S_)
            D = dy[sl].reshape(-1, C, S_)
            return (np.sum(D * (X - m32[None, :, None]), axis=(0, 2), dtype=np.float64),
                    np.sum(D, axis=(0, 2), dtype=np.float64))
        parts = list(pool.map(red, nch))
        rstd = (F32(1.0) / np.sqrt(v32 + eps)).astype(F32)
        dg = (sum(p[0] for p in parts) * rstd).astype(F32)
        db = sum(p[1] for p in parts).astype(F32)

        def bwd(s):
            sl = slice(s[0] * plane, s[1] * plane)
            return S.batchnorm_backward_dx(x[sl], dy[sl], m32, v32, gamma, dg, db, s[1] - s[0], C, S_, eps,
                                           count=cnt)
        list(pool.map(bwd, nch))
    secs, n = _timed(step, reps, min_seconds)
    pool.shutdown()
    nbytes = 4 * 3 * N * plane + 4 * 5 * N * plane
    desc = f"C5b sample: x[{N},{C},56,56] (1/{256 // N} of the batch), BN train fwd+bwd; {n} passes, {threads} threads"
    return nbytes / secs / 1e9, secs, desc
