"""The sharded (dct_dist_*) entry points on the GPU.

World size 1 (a one-rank NCCL communicator, always runnable): every sharded op
is bit-identical to its single-GPU entry point, which is itself held to the
oracle elsewhere (and here, for the BatchNorm extension entry points).  The
host-made failures: an inconsistent shard header makes the next wait return
DCT_ERR_DIST, and a device-side bounded wait that runs out makes it return
DCT_ERR_CUDA; the context stays usable after both.

World size 2 (only with two GPUs): two processes, one GPU each, shard the
rows / batch; every rank's result equals the unsharded oracle on the whole
input (bit-exact for max/min/argmax/argmin and the dlogits formula, rel 1e-5
for sums, means, losses and BatchNorm statistics).
"""
import datetime
import multiprocessing as mp
import os
import queue
import socket
import time
import traceback

import numpy as np
import pytest

from oracle import newops as O
from oracle import shaders as S

pytestmark = pytest.mark.gpu

REDUCE_OPS = ("sum", "mean", "max", "argmax", "min", "argmin", "sumsq")


def _same(a, b):
    a = np.asarray(a)
    b = np.asarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    av, bv = a.view(np.uint32), b.view(np.uint32)
    eq = (av == bv) | (np.isnan(a.view(np.float32)) & np.isnan(b.view(np.float32)))
    assert eq.all(), f"{(~eq).sum()} mismatches, first at {np.flatnonzero(~eq.ravel())[:5]}"


@pytest.fixture(scope="module")
def comm(dev):
    from directcompute_torch_b200.dist import Communicator
    c = Communicator.single(timeout_s=30)
    yield c
    c.close()


def _reduce_local(dev, op, hx, outer, n, inner, want_idx):
    lib = dev.lib
    hout = dev.empty(outer * inner)
    hidx = dev.empty(outer * inner) if want_idx else None
    from directcompute_torch_b200._abi import REDUCE
    assert lib.dct_reduce(REDUCE[op], hx, outer, n, inner, hout, hidx) == 0, dev.error()
    return hout, hidx


@pytest.mark.parametrize("shape", [(1, 1000, 4096), (1, 333, 37), (6, 40, 512), (64, 1, 1), (3, 100, 1)])
def test_world1_reduce_matches_local(dev, comm, shape):
    outer, n, inner = shape
    r = np.random.default_rng(31)
    x = r.standard_normal(shape).astype(np.float32)
    x.ravel()[r.choice(x.size, size=max(1, x.size // 500), replace=False)] = 1e4
    hx = dev.buf(x)
    for op in REDUCE_OPS:
        for want_idx in ((False, True) if op in ("max", "min", "argmax") else (False,)):
            ha, hai = _reduce_local(dev, op, hx, outer, n, inner, want_idx)
            hb = dev.empty(outer * inner)
            hbi = dev.empty(outer * inner) if want_idx else None
            comm.reduce(op, hx, outer, n, inner, 0, n, hb, hbi)
            dev.sync()
            _same(dev.read(hb), dev.read(ha))
            if want_idx:
                _same(dev.read(hbi), dev.read(hai))
            dev.free(ha, hb, *(h for h in (hai, hbi) if h))
    dev.free(hx)


def test_world1_reduce_all_matches_local(dev, comm):
    r = np.random.default_rng(32)
    for n in (1, 1000, (1 << 22) + 3):
        x = r.uniform(-1, 1, n).astype(np.float32)
        hx = dev.buf(x)
        for op in ("sum", "mean", "max", "min", "sumsq"):
            ha, hb = dev.empty(1), dev.empty(1)
            va = dev.reduce_all(op, hx, n, ha)
            vb = comm.reduce_all(op, hx, n, hb, want_host=True)
            assert va == vb or (np.isnan(va) and np.isnan(vb)), (op, n, va, vb)
            _same(dev.read(hb), dev.read(ha))
            dev.free(ha, hb)
        dev.free(hx)


@pytest.mark.parametrize("BK", [(4096, 1000), (300, 37), (64, 3000)])
def test_world1_softmax_ce_matches_local(dev, comm, BK):
    B, K = BK
    r = np.random.default_rng(33)
    x = (3 * r.standard_normal((B, K))).astype(np.float32)
    lab = r.integers(0, K, B).astype(np.float32)
    hx, hl = dev.buf(x), dev.buf(lab)
    outs = []
    for sharded in (False, True):
        hp, hg, hloss = dev.empty(B * K), dev.empty(B * K), dev.empty(1)
        if sharded:
            comm.softmax_ce(hx, hl, B, K, probs=hp, dlogits=hg, loss=hloss, global_rows=B)
        else:
            assert dev.lib.dct_softmax_ce(hx, hl, 0, B, K, hp, hg, hloss, None, float(B), float(B)) == 0, dev.error()
        dev.sync()
        outs.append([dev.read(h) for h in (hp, hg, hloss)])
        dev.free(hp, hg, hloss)
    for a, b in zip(*outs):
        _same(b, a)
    p, loss, _ = O.softmax_ce_f64(x, lab.astype(np.int64))
    assert abs(float(outs[1][2][0]) - float(loss)) <= 1e-5 * abs(float(loss))
    dev.free(hx, hl)


def _bn_inputs(shape, seed):
    r = np.random.default_rng(seed)
    N, C, H, W = shape
    x = (0.5 + 2 * r.standard_normal(shape)).astype(np.float32)
    dy = r.standard_normal(shape).astype(np.float32)
    gamma = r.random(C, dtype=np.float32)
    beta = r.random(C, dtype=np.float32)
    rm0 = (0.1 * r.standard_normal(C)).astype(np.float32)
    rv0 = (1.0 + r.random(C, dtype=np.float32)).astype(np.float32)
    return x, dy, gamma, beta, rm0, rv0


def _bn_dx_global(x, dy, mean, var, gamma, dg, db, C, S_, m_count, eps):
    """nn_batchnorm_backward_dx.hlsl:20-38 with m = the global element count per channel."""
    n = x.size
    c = (np.arange(n, dtype=np.int64) // S_) % C
    rstd = (np.float32(1.0) / np.sqrt(var[:C] + np.float32(eps))).astype(np.float32)
    xhat = ((x.ravel() - mean[c]) * rstd[c]).astype(np.float32)
    inner = ((db[c] + xhat * dg[c]) / np.float32(m_count)).astype(np.float32)
    return ((gamma[c] * rstd[c]) * (dy.ravel() - inner)).astype(np.float32)


@pytest.mark.parametrize("shape", [(8, 16, 7, 7), (16, 64, 28, 28), (3, 5, 3, 3)])
def test_world1_batchnorm_matches_local_and_oracle(dev, comm, shape):
    N, C, H, W = shape
    S_ = H * W
    eps = 1e-5
    x, dy, gamma, beta, rm0, rv0 = _bn_inputs(shape, 34)
    hx, hdy, hg, hb = dev.buf(x), dev.buf(dy), dev.buf(gamma), dev.buf(beta)
    res = []
    lib = dev.lib
    for sharded in (False, True):
        hrm, hrv, hm, hv, hy = dev.buf(rm0), dev.buf(rv0), dev.empty(C), dev.empty(C), dev.empty(x.size)
        hdg, hdb, hdx = dev.empty(C), dev.empty(C), dev.empty(x.size)
        if sharded:
            comm.batchnorm_forward_train(hx, hg, hb, hrm, hrv, hm, hv, hy, N, C, S_, eps, 0.1)
            comm.batchnorm_backward(hx, hdy, hm, hv, hg, hdg, hdb, hdx, N, C, S_, eps)
        else:
            assert lib.dct_batchnorm_forward_train(hx, hg, hb, hrm, hrv, hm, hv, hy, N, C, S_, eps, 0.1) == 0
            assert lib.dct_batchnorm_backward(hx, hdy, hm, hv, hg, hdg, hdb, hdx, N, C, S_, eps) == 0
        dev.sync()
        res.append([dev.read(h) for h in (hrm, hrv, hm, hv, hy, hdg, hdb, hdx)])
        dev.free(hrm, hrv, hm, hv, hy, hdg, hdb, hdx)
    for a, b in zip(*res):
        _same(b, a)
    rm, rv, mean, var, y, dg, db, dx = res[1]
    mean64, var64 = S.batchnorm_mean_var(x.ravel(), N, C, S_)
    assert np.allclose(mean, mean64, rtol=1e-6, atol=1e-7) and np.allclose(var, var64, rtol=1e-6)
    rm_o, rv_o = S.batchnorm_running(rm0, rv0, mean64, var64, N, S_, 0.1)
    assert np.allclose(rm, rm_o, rtol=1e-6, atol=1e-8) and np.allclose(rv, rv_o, rtol=1e-6)
    _same(y, S.batchnorm_forward(x.ravel(), mean, var, gamma, beta, N, C, S_, np.float32(eps)))
    dg_o, db_o = S.batchnorm_backward_reduce(x.ravel(), dy.ravel(), mean, var, N, C, S_, np.float32(eps))
    tol = 1e-6 * np.sqrt(N * S_)
    assert np.allclose(dg, dg_o, rtol=1e-5, atol=tol) and np.allclose(db, db_o, rtol=1e-5, atol=tol)
    _same(dx, S.batchnorm_backward_dx(x.ravel(), dy.ravel(), mean, var, gamma, dg, db, N, C, S_, np.float32(eps)))
    dev.free(hx, hdy, hg, hb)


def test_world1_allreduce_broadcast_barrier(dev, comm):
    v = np.arange(1000, dtype=np.float32) - 300.5
    h = dev.buf(v)
    for op in ("sum", "mean", "max", "min"):
        comm.allreduce(h, v.size, op)
    comm.broadcast(h, v.size, 0)
    comm.barrier()
    _same(dev.read(h), v)
    dev.free(h)


def test_world1_inconsistent_shards_fail_on_every_wait(dev, comm):
    """A shard header that does not tile [0, len_total) is caught on the device."""
    x = np.ones((1, 100, 8), np.float32)
    hx, ho = dev.buf(x), dev.empty(8)
    comm.reduce("sum", hx, 1, 100, 8, 0, 200, ho)          # claims a 200-row axis, holds 100 rows
    rc = dev.lib.dct_synchronize()
    code, msg = dev.error()
    assert rc == 8 and code == 8 and "shard" in msg, (rc, code, msg)
    dev.clear_error()
    comm.reduce("sum", hx, 1, 100, 8, 0, 100, ho)          # the same call, consistent: fine
    dev.sync()
    _same(dev.read(ho), np.full(8, 100.0, np.float32))
    dev.free(hx, ho)


def test_bounded_wait_times_out_and_context_survives(dev):
    """A kernel waits on a barrier phase that nothing completes; the wait gives
    up after its poll budget, reports through the error word, and the next op works."""
    lib = dev.lib
    dev.sync()
    t0 = time.perf_counter()
    assert lib.dct_selftest_bounded_wait(4096) == 0, dev.error()
    rc = lib.dct_synchronize()
    secs = time.perf_counter() - t0
    code, msg = dev.error()
    assert rc == 5 and code == 5 and "bounded wait" in msg, (rc, code, msg)
    assert secs < 30, secs
    dev.clear_error()
    a = np.arange(4096, dtype=np.float32)
    ha, hb = dev.buf(a), dev.empty(a.size)
    dev.unary("neg", ha, hb, a.size)
    dev.sync()
    _same(dev.read(hb), -a)
    dev.free(ha, hb)
    print(f"bounded wait of 4096 polls gave up after {secs * 1e3:.1f} ms (host-observed)")


def _lonely_rank(q):
    """Rank 0 of a 2-rank communicator that rank 1 never joins (one GPU, one process)."""
    try:
        import torch  # noqa: F401
        from directcompute_torch_b200 import load_library
        from directcompute_torch_b200.dist import Communicator
        lib = load_library()
        assert lib.InitEngine()
        t0 = time.monotonic()
        try:
            Communicator(0, 2, Communicator.new_unique_id(), timeout_s=3)
            q.put(("returned", time.monotonic() - t0, ""))
        except RuntimeError as e:
            q.put(("raised", time.monotonic() - t0, str(e)))
        # work on the device still runs after the failed init
        h = lib.dct_create_buffer(1024)
        lib.ClearBuffer(h)
        q.put(("sync", lib.dct_synchronize(), ""))
    except BaseException:
        q.put(("crash", 0.0, traceback.format_exc()))
    q.close()
    q.join_thread()    # flush the queue's feeder thread before leaving
    os._exit(0)        # the abandoned init helper is still waiting for rank 1: skip exit-time teardown


def test_init_gives_up_when_a_rank_never_joins():
    """Host-made failure: the peer never calls init.  dct_dist_init returns
    DCT_ERR_DIST at its deadline instead of blocking the caller."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(q,))
    p.start()
    try:
        what, secs, msg = q.get(timeout=120)
        assert what == "raised", (what, msg)
        assert "not every rank joined" in msg and 2.5 < secs < 30, (secs, msg)
        what, rc, msg = q.get(timeout=60)
        assert what == "sync" and rc == 0, (what, rc, msg)
    finally:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()


# ---------------------------------------------------------------------------
# one process per visible GPU (2 to 8)
# ---------------------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _collect(q, procs, limit_s):
    """Every rank's (ok, payload) from q.  A rank whose process ended without
    posting (a crash) fails the test at once, with the others' reports."""
    res, deadline = {}, time.monotonic() + limit_s
    while len(res) < len(procs):
        try:
            r, ok, payload = q.get(timeout=5)
            res[r] = (ok, payload)
            continue
        except queue.Empty:
            pass
        dead = [i for i, p in enumerate(procs) if i not in res and p.exitcode not in (None, 0)]
        if dead or time.monotonic() > deadline:
            while True:                          # reports already queued
                try:
                    r, ok, payload = q.get(timeout=1)
                    res[r] = (ok, payload)
                except queue.Empty:
                    break
            missing = [i for i in range(len(procs)) if i not in res]
            raise AssertionError(f"ranks {missing} posted nothing (exit codes "
                                 f"{[procs[i].exitcode for i in missing]}); reports: {res}")
    return res


def _worldn_worker(rank, world, port, q, transport="peer"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), DCT_DEVICE=str(rank),
                      NCCL_NVLS_ENABLE="0", DCT_PEER_EXCHANGE="0" if transport == "nccl" else "1")
    try:
        import torch  # noqa: F401  (loads PyTorch's NCCL first)
        import torch.distributed as td
        td.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from tests.devhelp import Dev
        from directcompute_torch_b200.dist import Communicator, shard_range
        dev = Dev()
        comm = Communicator.from_process_group(timeout_s=60)
        errs = {"peer_exchange": comm.peer_exchange}
        r = np.random.default_rng(40)
        # C3-style axis-0 reductions, rows sharded (uneven split)
        R, Cc = 1001, 640
        x = r.standard_normal((R, Cc)).astype(np.float32)
        x[r.integers(0, R, 50), r.integers(0, Cc, 50)] = 1e4
        b = shard_range(R, world, 1)[0]
        x[b - 1, 5] = x[b, 5] = 2e4                        # tie across the boundary
        x[b + 3, 7] = np.nan
        off, cnt = shard_range(R, world, rank)
        hx = dev.buf(x[off:off + cnt])
        for op in ("sum", "mean", "max", "argmax", "min", "argmin"):
            ho = dev.empty(Cc)
            comm.reduce(op, hx, 1, cnt, Cc, off, R, ho)
            dev.sync()
            got = dev.read(ho, np.int32 if op.startswith("arg") else np.float32)
            want = O.reduce(op, x, axis=0)
            if op in ("sum", "mean"):
                # a true relative bound on the float64-accumulated result, plus the float64
                # accumulation's own noise (1e-12 of sum|x|) where the column nearly cancels
                x64 = x.astype(np.float64)
                want = x64.sum(axis=0) / (1 if op == "sum" else R)
                mag = np.abs(x64).sum(axis=0) / (1 if op == "sum" else R)
                fin = np.isfinite(want)
                err = np.abs(got[fin] - want[fin])
                errs[op] = float(np.max(np.maximum(err - 1e-12 * mag[fin], 0.0) / np.abs(want[fin])))
            else:
                errs[op] = int(np.sum(~((got == want) | (np.isnan(got.astype(np.float32)) & np.isnan(
                    want.astype(np.float32))))))
            dev.free(ho)
        dev.free(hx)
        # small shards: a single-chunk plan (its record staged, then the separate
        # put/wait/fold kernel) and, with fewer rows than ranks, an empty shard
        for R2 in (2 * world, world - 1):
            x2 = r.standard_normal((R2, 96)).astype(np.float32)
            o5, c5 = shard_range(R2, world, rank)
            hx2 = dev.buf(x2[o5:o5 + c5]) if c5 else dev.empty(1)
            for op in ("sum", "max", "argmax"):
                ho = dev.empty(96)
                comm.reduce(op, hx2, 1, c5, 96, o5, R2, ho)
                dev.sync()
                got = dev.read(ho, np.int32 if op == "argmax" else np.float32)
                if op == "sum":
                    x64 = x2.astype(np.float64)
                    want, mag = x64.sum(axis=0), np.abs(x64).sum(axis=0)
                    err = np.maximum(np.abs(got - want) - 1e-12 * mag, 0.0) / np.abs(want)
                    errs[f"small{R2}_sum"] = float(np.max(err))
                else:
                    errs[f"small{R2}_{op}"] = int(np.sum(got != O.reduce(op, x2, axis=0)))
                dev.free(ho)
            dev.free(hx2)
            v2 = r.uniform(-1, 1, R2).astype(np.float32)
            hv2, ho2 = (dev.buf(v2[o5:o5 + c5]) if c5 else dev.empty(1)), dev.empty(1)
            s2 = comm.reduce_all("sum", hv2, c5, ho2, want_host=True)
            want2 = float(v2.astype(np.float64).sum())
            errs[f"small{R2}_full_sum"] = abs(s2 - want2) / max(abs(want2), 1e-30)
            errs[f"small{R2}_full_max"] = int(comm.reduce_all("max", hv2, c5, ho2, want_host=True) != float(v2.max()))
            dev.free(hv2, ho2)
        # full reduction of a flat vector
        n = (1 << 21) + 5
        v = r.uniform(-1, 1, n).astype(np.float32)
        o2, c2 = shard_range(n, world, rank)
        hv, ho = dev.buf(v[o2:o2 + c2]), dev.empty(1)
        s = comm.reduce_all("sum", hv, c2, ho, want_host=True)
        errs["full_sum"] = abs(s - float(v.astype(np.float64).sum())) / abs(float(v.astype(np.float64).sum()))
        mx = comm.reduce_all("max", hv, c2, ho, want_host=True)
        errs["full_max"] = int(mx != float(v.max()))
        dev.free(hv, ho)
        # softmax + CE, rows sharded, global divisor
        B, K = 3000, 1000
        lg = (3 * r.standard_normal((B, K))).astype(np.float32)
        lab = r.integers(0, K, B)
        o3, c3 = shard_range(B, world, rank)
        hl, ht = dev.buf(lg[o3:o3 + c3]), dev.buf(lab[o3:o3 + c3].astype(np.float32))
        hp, hg, hloss = dev.empty(c3 * K), dev.empty(c3 * K), dev.empty(1)
        comm.softmax_ce(hl, ht, c3, K, probs=hp, dlogits=hg, loss=hloss, global_rows=B)
        dev.sync()
        _, loss64, _ = O.softmax_ce_f64(lg, lab)
        errs["loss"] = abs(float(dev.read(hloss)[0]) - float(loss64)) / abs(float(loss64))
        p_dev = dev.read(hp).reshape(c3, K)
        want_g = O.softmax_ce_dlogits(p_dev, lab[o3:o3 + c3], B)
        errs["dlogits"] = int(np.sum(dev.read(hg).view(np.uint32) != want_g.ravel().view(np.uint32)))
        dev.free(hl, ht, hp, hg, hloss)
        # BatchNorm, batch sharded
        shape = (10, 32, 14, 14)
        N, C, H, W = shape
        S_ = H * W
        x, dy, gamma, beta, rm0, rv0 = _bn_inputs(shape, 41)
        o4, c4 = shard_range(N, world, rank)
        hx, hdy = dev.buf(x[o4:o4 + c4]), dev.buf(dy[o4:o4 + c4])
        hgm, hbt, hrm, hrv = dev.buf(gamma), dev.buf(beta), dev.buf(rm0), dev.buf(rv0)
        hm, hvv, hy = dev.empty(C), dev.empty(C), dev.empty(c4 * C * S_)
        hdg, hdb, hdx = dev.empty(C), dev.empty(C), dev.empty(c4 * C * S_)
        comm.batchnorm_forward_train(hx, hgm, hbt, hrm, hrv, hm, hvv, hy, c4, C, S_, 1e-5, 0.1)
        comm.batchnorm_backward(hx, hdy, hm, hvv, hgm, hdg, hdb, hdx, c4, C, S_, 1e-5)
        dev.sync()
        mean64, var64 = S.batchnorm_mean_var(x.ravel(), N, C, S_)
        mean, var = dev.read(hm), dev.read(hvv)
        errs["bn_mean"] = float(np.max(np.abs(mean - mean64) / np.maximum(np.abs(mean64), 1e-3)))
        errs["bn_var"] = float(np.max(np.abs(var - var64) / var64))
        rm_o, rv_o = S.batchnorm_running(rm0, rv0, mean64, var64, N, S_, 0.1)
        errs["bn_running"] = float(max(np.max(np.abs(dev.read(hrm) - rm_o)), np.max(np.abs(dev.read(hrv) - rv_o) / rv_o)))
        y_o = S.batchnorm_forward(x[o4:o4 + c4].ravel(), mean, var, gamma, beta, c4, C, S_, np.float32(1e-5))
        errs["bn_y"] = int(np.sum(dev.read(hy).view(np.uint32) != y_o.view(np.uint32)))
        dg_o, db_o = S.batchnorm_backward_reduce(x.ravel(), dy.ravel(), mean, var, N, C, S_, np.float32(1e-5))
        dg, db = dev.read(hdg), dev.read(hdb)
        errs["bn_dgamma"] = float(np.max(np.abs(dg - dg_o) / np.maximum(np.abs(dg_o), np.sqrt(N * S_) * 1e-6)))
        errs["bn_dbeta"] = float(np.max(np.abs(db - db_o) / np.maximum(np.abs(db_o), np.sqrt(N * S_) * 1e-6)))
        dx_o = _bn_dx_global(x[o4:o4 + c4], dy[o4:o4 + c4], mean, var, gamma, dg, db, C, S_, N * S_, 1e-5)
        errs["bn_dx"] = int(np.sum(dev.read(hdx).view(np.uint32) != dx_o.view(np.uint32)))
        dev.free(hx, hdy, hgm, hbt, hrm, hrv, hm, hvv, hy, hdg, hdb, hdx)
        # an empty rank (fewer rows / samples than ranks): softmax-CE and BatchNorm
        B2, K2 = world - 1, 64
        lg2 = (3 * r.standard_normal((B2, K2))).astype(np.float32)
        lab2 = r.integers(0, K2, B2)
        o6, c6 = shard_range(B2, world, rank)
        hl2 = dev.buf(lg2[o6:o6 + c6]) if c6 else dev.empty(1)
        ht2 = dev.buf(lab2[o6:o6 + c6].astype(np.float32)) if c6 else dev.empty(1)
        hp2, hg2, hs2 = dev.empty(max(c6, 1) * K2), dev.empty(max(c6, 1) * K2), dev.empty(1)
        comm.softmax_ce(hl2, ht2, c6, K2, probs=hp2, dlogits=hg2, loss=hs2, global_rows=B2)
        dev.sync()
        _, l64, _ = O.softmax_ce_f64(lg2, lab2)
        errs["small_loss"] = abs(float(dev.read(hs2)[0]) - float(l64)) / abs(float(l64))
        dev.free(hl2, ht2, hp2, hg2, hs2)
        shape2 = (world - 1, 4, 3, 3)
        N2, C2 = shape2[0], shape2[1]
        S2 = shape2[2] * shape2[3]
        xb, dyb, gb, bb, rmb, rvb = _bn_inputs(shape2, 42)
        o7, c7 = shard_range(N2, world, rank)
        hx = dev.buf(xb[o7:o7 + c7]) if c7 else dev.empty(1)
        hgm, hbt, hrm, hrv = dev.buf(gb), dev.buf(bb), dev.buf(rmb), dev.buf(rvb)
        hm, hvv, hy = dev.empty(C2), dev.empty(C2), dev.empty(max(c7, 1) * C2 * S2)
        comm.batchnorm_forward_train(hx, hgm, hbt, hrm, hrv, hm, hvv, hy, c7, C2, S2, 1e-5, 0.1)
        dev.sync()
        m64, v64 = S.batchnorm_mean_var(xb.ravel(), N2, C2, S2)
        errs["small_bn_mean"] = float(np.max(np.abs(dev.read(hm) - m64) / np.maximum(np.abs(m64), 1e-3)))
        errs["small_bn_var"] = float(np.max(np.abs(dev.read(hvv) - v64) / v64))
        dev.free(hx, hgm, hbt, hrm, hrv, hm, hvv, hy)
        # fp32 all-reduce
        a = np.full(4099, rank + 1.0, np.float32)
        ha = dev.buf(a)
        comm.allreduce(ha, a.size, "sum")
        dev.sync()
        errs["allreduce"] = int(np.sum(dev.read(ha) != sum(range(1, world + 1))))
        dev.free(ha)
        comm.close()
        td.destroy_process_group()
        q.put((rank, True, errs))
    except BaseException:
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.parametrize("transport", ["peer", "nccl"])
def test_worldn_sharded_ops_match_unsharded_oracle(transport):
    """Every visible GPU (2 to 8) as one rank: the sharded ops, over the peer-memory
    exchange and over the NCCL all-gather fallback, match the oracle on the unsharded
    tensors."""
    import torch
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worldn_worker, args=(r, world, port, q, transport)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = _collect(q, procs, 600)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        ok, e = res[r]
        assert ok, e
        print(f"rank {r}: {e}")
        assert e["peer_exchange"] == (transport == "peer"), (r, transport)
        small = [f"small{R2}_" for R2 in (2 * world, world - 1)]
        for k in ("max", "argmax", "min", "argmin", "full_max", "dlogits", "bn_y", "bn_dx", "allreduce",
                  *[p + q for p in small for q in ("max", "argmax", "full_max")]):
            assert e[k] == 0, (r, k, e[k])
        for k in ("sum", "mean", "full_sum", "loss", "bn_mean", "bn_var", "bn_running", "bn_dgamma", "bn_dbeta",
                  *[p + q for p in small for q in ("sum", "full_sum")], "small_loss", "small_bn_mean",
                  "small_bn_var"):
            assert e[k] <= 1e-5, (r, k, e[k])


# ---------------------------------------------------------------------------
# a live rank that skips one exchange (two GPUs): the bounded device wait
# ---------------------------------------------------------------------------
def _skip_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), DCT_DEVICE=str(rank),
                      NCCL_NVLS_ENABLE="0", DCT_PEER_EXCHANGE="1")
    try:
        import torch  # noqa: F401  (loads PyTorch's NCCL first)
        import torch.distributed as td
        td.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        from tests.devhelp import Dev
        from directcompute_torch_b200.dist import Communicator
        dev = Dev()
        comm = Communicator.from_process_group(timeout_s=3)
        out = {"peer": comm.peer_exchange}
        v = np.ones(4096, np.float32)
        hv, ho = dev.buf(v), dev.empty(1)
        out["warm"] = comm.reduce_all("sum", hv, v.size, ho, want_host=True)     # every rank takes part
        td.barrier()
        if rank == 0:                         # rank 1 stays alive but skips this exchange
            t0 = time.monotonic()
            try:
                comm.reduce_all("sum", hv, v.size, ho, want_host=True)
                out["missed"] = None
            except RuntimeError as e:
                out["missed"] = str(e)
            out["secs"] = time.monotonic() - t0
        td.barrier()
        # teardown without any kernel of ours in flight: the rank whose communicator
        # was aborted closes its mappings first, then the other finalizes (its closing
        # barrier over NCCL ends at the 3 s limit, since rank 0's communicator is gone)
        for turn in range(world):
            if rank == turn:
                try:
                    comm.close()
                    out["close"] = "ok"
                except RuntimeError as e:
                    out["close"] = str(e)
            td.barrier()
        out["after"] = dev.reduce_all("sum", hv, v.size, ho)                      # the context still works
        dev.free(hv, ho)
        td.destroy_process_group()
        q.put((rank, True, out))
    except BaseException:
        q.put((rank, False, traceback.format_exc()))


def test_worldn_peer_wait_times_out_when_a_rank_skips_an_exchange():
    """Two GPUs over the peer-memory exchange, timeout 3 s: rank 1 stays alive but
    skips one dct_dist_reduce_all.  Rank 0's exchange kernel gives up at its bounded
    %globaltimer wait and returns DCT_ERR_DIST naming the missing record, within the
    limit; both ranks then close their communicators and keep a usable context."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_skip_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = _collect(q, procs, 300)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        ok, e = res[r]
        assert ok, e
        print(f"rank {r}: {e}")
        assert e["warm"] == 2 * 4096.0 and e["after"] == 4096.0, e
        if not e["peer"]:
            pytest.skip("the peer-memory exchange is not available between these GPUs")
    e0 = res[0][1]
    assert e0["missed"] is not None and "DIST" in e0["missed"] and "did not arrive" in e0["missed"], e0
    assert 1.0 < e0["secs"] < 15.0, e0
