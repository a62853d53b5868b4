"""Host-side logic of the multi-GPU path, on CPU ranks over `gloo` (world size 2).

* the shard split: Python (`dist.shard_range`), the library (`dct_dist_shard`,
  no device needed) and the oracle agree and tile the axis;
* the combine rule: each rank reduces its shard to the partial the library
  exchanges, the partials travel over gloo, the rank-order fold equals the
  unsharded NumPy-semantics oracle (bit-exact for max/min/argmax/argmin, with
  ties and NaNs placed across the shard boundary);
* the NCCL unique-id exchange over a torch.distributed group, and the quiet
  DCT_ERR_NO_DEVICE failure of dct_dist_init on a machine without a GPU;
* failure detection on the host: a rank that dies before the exchange makes
  the other rank's exchange raise within the group timeout instead of hanging.
"""
import ctypes
import datetime
import multiprocessing as mp
import os
import socket
import traceback

import numpy as np
import pytest

from oracle import newops, sharded

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(target, world=WORLD, timeout=120, **kw):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(target, r, world, port, q, kw)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, ok, payload = q.get(timeout=timeout)
            res[r] = (ok, payload)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return res


def _entry(target, rank, world, port, q, kw):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        import torch.distributed as td
        td.init_process_group("gloo", rank=rank, world_size=world,
                              timeout=datetime.timedelta(seconds=kw.pop("pg_timeout", 60)))
        try:
            payload = globals()[target](rank, world, **kw)
            q.put((rank, True, payload))
        finally:
            try:
                td.destroy_process_group()
            except Exception:
                pass
    except BaseException:
        q.put((rank, False, traceback.format_exc()))


# ---------------------------------------------------------------------------
def test_shard_range_matches_library():
    from directcompute_torch_b200 import dist, load_library
    lib = load_library()
    off, cnt = ctypes.c_uint64(), ctypes.c_uint64()
    for n in list(range(0, 40)) + [16384, 2**30 + 7]:
        for world in range(1, 9):
            pos = 0
            for r in range(world):
                assert lib.dct_dist_shard(n, world, r, ctypes.byref(off), ctypes.byref(cnt)) == 0
                assert (off.value, cnt.value) == dist.shard_range(n, world, r) == sharded.shard_range(n, world, r)
                assert off.value == pos
                pos += cnt.value
            assert pos == n
            counts = [dist.shard_range(n, world, r)[1] for r in range(world)]
            assert max(counts) - min(counts) <= 1
    assert lib.dct_dist_shard(10, 0, 0, ctypes.byref(off), ctypes.byref(cnt)) != 0
    assert lib.dct_dist_shard(10, 2, 2, ctypes.byref(off), ctypes.byref(cnt)) != 0


def _axis_case():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((3, 37, 6)).astype(np.float32)
    b = sharded.shard_range(37, WORLD, 1)[0]          # first row of rank 1
    x[0, b - 1, 0] = x[0, b, 0] = 50.0                 # tie straddling the boundary -> lower index
    x[1, b + 2, 1] = np.nan                            # NaN only in rank 1's shard
    x[1, 3, 1] = 99.0
    x[2, :, 2] = -1.0                                  # all equal -> index 0
    x[0, b, 3] = -77.0                                 # min right at the boundary
    return x


def _axis_worker(rank, world):
    import torch.distributed as td
    x = _axis_case()
    off, cnt = sharded.shard_range(x.shape[1], world, rank)
    out = {}
    for op in ("sum", "mean", "max", "argmax", "min", "argmin"):
        part = sharded.axis_partial(op, x[:, off:off + cnt, :], off)
        gathered = [None] * world
        td.all_gather_object(gathered, part)
        out[op] = sharded.fold_axis(op, gathered, x.shape[1])
    for op in ("sum", "mean", "max", "min", "sumsq"):
        part = sharded.full_partial(op, x.ravel()[sharded.shard_range(x.size, world, rank)[0]:][
            :sharded.shard_range(x.size, world, rank)[1]])
        gathered = [None] * world
        td.all_gather_object(gathered, part)
        out["full_" + op] = sharded.fold_full(op, gathered)
    return out


def test_gloo_sharded_fold_matches_unsharded():
    res = _run("_axis_worker")
    x = _axis_case()
    for r in range(WORLD):
        ok, payload = res[r]
        assert ok, payload
        for op in ("max", "argmax", "min", "argmin"):
            np.testing.assert_array_equal(payload[op], newops.reduce(op, x, axis=1))
        for op in ("sum", "mean"):
            np.testing.assert_allclose(payload[op], newops.reduce(op, x, axis=1), rtol=1e-6, atol=1e-6)
        x64 = x.astype(np.float64).ravel()
        np.testing.assert_allclose(payload["full_sum"], x64.sum(), rtol=1e-12)
        np.testing.assert_allclose(payload["full_mean"], x64.mean(), rtol=1e-12)
        np.testing.assert_allclose(payload["full_sumsq"], (x64 ** 2).sum(), rtol=1e-12)
        assert np.isnan(payload["full_max"]) and np.isnan(payload["full_min"])   # one NaN anywhere
    # both ranks hold the same result
    for op in res[0][1]:
        np.testing.assert_array_equal(np.asarray(res[0][1][op]), np.asarray(res[1][1][op]))


def _id_worker(rank, world):
    from directcompute_torch_b200.dist import Communicator
    r, w, uid = Communicator.exchange_id()
    init_error = None
    try:
        Communicator(r, w, uid, timeout_s=10).close()
    except RuntimeError as e:
        init_error = str(e)
    return {"rank": r, "world": w, "uid": uid, "init_error": init_error}


def test_gloo_nccl_id_exchange_and_quiet_init_failure():
    from directcompute_torch_b200 import dist
    if not dist.nccl_available():
        pytest.skip("no NCCL library to make an id with")
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the no-device failure path does not apply")
    res = _run("_id_worker")
    uids = []
    for r in range(WORLD):
        ok, p = res[r]
        assert ok, p
        assert p["rank"] == r and p["world"] == WORLD and len(p["uid"]) == 128
        assert p["init_error"] is not None and "NO_DEVICE" in p["init_error"]
        uids.append(p["uid"])
    assert uids[0] == uids[1] and any(uids[0])


def _dying_worker(rank, world):
    from directcompute_torch_b200.dist import Communicator
    if rank == 1:
        os._exit(3)                                    # leaves without joining the exchange
    import time
    t0 = time.monotonic()
    try:
        Communicator.exchange_id()
    except Exception as e:                             # the peer is gone: must raise, not hang
        return {"raised": type(e).__name__, "secs": time.monotonic() - t0}
    return {"raised": None, "secs": time.monotonic() - t0}


def test_gloo_dead_rank_is_detected_not_hung():
    from directcompute_torch_b200 import dist
    if not dist.nccl_available():
        pytest.skip("no NCCL library to make an id with")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=("_dying_worker", r, WORLD, port, q, {"pg_timeout": 5}))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        r, ok, payload = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert r == 0 and ok, payload
    assert payload["raised"] is not None, "the exchange with a dead rank returned normally"
    assert payload["secs"] < 60
