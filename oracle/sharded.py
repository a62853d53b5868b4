"""Combine rules of the sharded ops -- TEST INFRASTRUCTURE ONLY.

The reference has one device and no multi-GPU path, so a sharded op is correct
when it returns what the unsharded NumPy-semantics oracle (`newops.reduce`,
`newops.softmax_ce_f64`, `shaders.batchnorm_*`) returns on the concatenation
of the shards.  This module states, on the CPU, the partial each rank produces
and the rank-order fold that libdct_cuda's dct_dist_* entry points perform on
the device:

* sums / means: float64 partial sum of the shard; partials added in rank
  order; a mean divides by the global extent;
* max / min: NaN if the shard holds a NaN, else the extreme; NaN wins the fold;
* argmax / argmin: (value, global index) of the shard's first best element
  (NaN first); the fold keeps the better value, ties and NaNs to the lower
  index, which is NumPy's first-occurrence rule on the whole axis;
* a shard with nothing to reduce contributes the identity (no candidate).

The CPU tests run this over `gloo` ranks and check fold(shards) against the
unsharded oracle; the GPU tests hold the device to the unsharded oracle.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
F64 = np.float64


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """The library's balanced contiguous split (dct_dist_shard)."""
    base, rem = divmod(n, world)
    return rank * base + min(rank, rem), base + (1 if rank < rem else 0)


def _best(op, vals, idxs):
    """First-best element of 1-D candidates under NumPy's rule (NaN first, lowest index)."""
    is_max = op in ("max", "argmax")
    best_v, best_i = None, -1
    for v, i in zip(vals, idxs):
        if i < 0:
            continue
        if best_i < 0:
            best_v, best_i = v, i
            continue
        vn, bn = np.isnan(v), np.isnan(best_v)
        if vn or bn:
            take = (vn and not bn) or (vn and bn and i < best_i)
        elif v != best_v:
            take = (v > best_v) if is_max else (v < best_v)
        else:
            take = i < best_i
        if take:
            best_v, best_i = v, i
    return best_v, best_i


def axis_partial(op: str, x: np.ndarray, offset: int):
    """Partial of one shard x[outer, len, inner] (len may be 0) whose rows start at `offset`.

    Returns a float64 array [outer, inner] for sums, else (values f32, global int64 indices)."""
    x = np.asarray(x, dtype=F32)
    outer, n, inner = x.shape
    if op in ("sum", "mean"):
        return x.astype(F64).sum(axis=1)
    vals = np.zeros((outer, inner), F32)
    idxs = np.full((outer, inner), -1, np.int64)
    if n == 0:
        return vals, idxs
    for o in range(outer):
        for c in range(inner):
            v, i = _best(op, x[o, :, c], np.arange(n))
            vals[o, c], idxs[o, c] = v, i + offset
    return vals, idxs


def fold_axis(op: str, partials, len_total: int):
    """Rank-order fold of `axis_partial` results -> the reduction of the whole axis."""
    if op in ("sum", "mean"):
        acc = partials[0].copy()
        for p in partials[1:]:
            acc = acc + p
        if op == "mean":
            acc = acc / F64(len_total)
        return acc.astype(F32)
    outer, inner = partials[0][0].shape
    out_v = np.zeros((outer, inner), F32)
    out_i = np.zeros((outer, inner), np.int32)
    for o in range(outer):
        for c in range(inner):
            v, i = _best(op, [p[0][o, c] for p in partials], [p[1][o, c] for p in partials])
            out_v[o, c], out_i[o, c] = v, i
    return out_i if op in ("argmax", "argmin") else out_v


def full_partial(op: str, x: np.ndarray):
    """(float64 value, count) of one shard of a full reduction (sum / mean / max / min / sumsq)."""
    x = np.asarray(x, dtype=F32).ravel()
    if op in ("sum", "mean"):
        return float(x.astype(F64).sum()), x.size
    if op == "sumsq":
        return float((x.astype(F64) ** 2).sum()), x.size
    if x.size == 0:
        return 0.0, 0
    if np.isnan(x).any():
        return float("nan"), x.size
    return float(x.max() if op == "max" else x.min()), x.size


def fold_full(op: str, partials) -> float:
    n = sum(c for _, c in partials)
    if op in ("sum", "mean", "sumsq"):
        acc = partials[0][0]
        for v, _ in partials[1:]:
            acc += v
        return acc / n if op == "mean" else acc
    cands = [v for v, c in partials if c > 0]
    if any(np.isnan(v) for v in cands):
        return float("nan")
    return max(cands) if op == "max" else min(cands)
