"""Replay of the reference's own engine calls (tests/golden/ref_trace.npz) through libdct_cuda.so.

The fixture was recorded from the unmodified reference `nn_engine.py` (see
tests/golden/make_golden.py).  Every dispatch is replayed alone: the same
shader name, the reference's cbuffer bytes and group counts, buffers of the
recorded sizes and contents (aliased where the reference aliased them), and
its UAVs compared with the recorded results.  Elementwise stages are
bit-exact (pooling indices bit for bit); sums and the loss rel 1e-5; softmax
4 ulp, sigmoid and the conv reshape's tanh 2 ulp (the HLSL intrinsics are
driver-defined); counts exact.  SGDBatch replays exactly;
SGDBatchClipped's norm and parameters rel 1e-6.
"""
import ctypes
import json
import os
import struct

import numpy as np
import pytest

from oracle.newops import ulp_diff

pytestmark = pytest.mark.gpu

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_trace.npz")
SUMS = {"loss", "bias_grad", "global_avg_pool", "batchnorm_mean_var", "batchnorm_backward_reduce", "dice_loss",
        "dice_loss_sums", "rms", "grad_sq_reduce", "grad_norm_final"}
ULPS = {"softmax": 4, "sigmoid": 2}
EXACT_BITS = {"maxpool_forward", "maxpool_backward"}       # index bits: no NaN-for-NaN matching


def _load():
    z = np.load(FIXTURE)
    return json.loads(str(z["meta"]))["records"], z


RECORDS, ARR = _load()


def _check(name, got, want, where, cb=b""):
    got = np.asarray(got, np.float32)
    want = np.asarray(want, np.float32)
    assert got.shape == want.shape, where
    if name == "conv_reshape" and len(cb) >= 20 and struct.unpack_from("<I", cb, 16)[0] == 2:
        nan = np.isnan(want)                                # tanh activation: 2 ulp
        assert np.array_equal(np.isnan(got), nan) and ulp_diff(got[~nan], want[~nan]).max() <= 2, where
    elif name in EXACT_BITS:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), where
    elif name in ULPS:
        assert ulp_diff(got, want).max() <= ULPS[name], where
    elif name in SUMS:
        g64, w64 = got.astype(np.float64), want.astype(np.float64)
        assert np.all(np.abs(g64 - w64) <= 1e-5 * np.abs(w64) + 1e-6), (where, np.abs(g64 - w64).max())
    else:
        eq = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
        assert eq.all(), f"{where}: {(~eq).sum()} mismatches, first at {np.flatnonzero(~eq)[:5]}"


def _replay_dispatch(dev, i, r):
    ids = {}
    handles = []

    def buf_for(hid, arr):
        if hid and hid in ids:
            return ids[hid]
        h = dev.buf(arr) if arr.size else dev.empty(1)
        handles.append(h)
        if hid:
            ids[hid] = h
        return h

    uavs = [buf_for(r["uav_ids"][j], ARR[f"r{i}_u{j}_in"]) for j in range(r["nuav"])]
    srvs = [buf_for(r["srv_ids"][j], ARR[f"r{i}_s{j}"]) for j in range(r["nsrv"])]
    dev.run(r["name"], srvs, uavs, tuple(r["groups"]), cb_bytes=bytes.fromhex(r["cb"]))
    code, msg = dev.error()
    assert code == 0, (i, r["name"], msg)
    for j in range(r["nuav"]):
        want = ARR[f"r{i}_u{j}_out"]
        got = dev.read(uavs[j])[: want.size]
        _check(r["name"], got, want, f"record {i} {r['name']} u{j}", bytes.fromhex(r["cb"]))
    dev.free(*handles)


def _replay_batch(dev, i, r):
    n, live = r["n"], r["live"]
    hp = [dev.buf(ARR[f"r{i}_p{j}_in"]) if j in live else None for j in range(n)]
    hg = [dev.buf(ARR[f"r{i}_g{j}"]) if j in live else None for j in range(n)]
    P = (ctypes.c_void_p * n)(*hp)
    G = (ctypes.c_void_p * n)(*hg)
    S = (ctypes.c_uint * n)(*r["sizes"])
    lib = dev.lib
    if r["kind"] == "SGDBatch":
        lib.SGDBatch(P, G, S, n, r["args"][0], r["args"][1])
        name = "sgd"
    else:
        norm = lib.SGDBatchClipped(P, G, S, n, r["args"][0], r["args"][1])
        assert abs(norm - r["ret"]) <= 1e-6 * abs(r["ret"]), (norm, r["ret"])
        name = "sgd_clipped"
    for j in live:
        want = ARR[f"r{i}_p{j}_out"]
        got = dev.read(hp[j])[: want.size]
        if name == "sgd":
            _check(name, got, want, f"record {i} SGDBatch p{j}")
        else:
            np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-7)
    dev.free(*(h for h in hp + hg if h))


@pytest.mark.parametrize("i", range(len(RECORDS)),
                         ids=[f"{k}-{r['name'] if r['kind'] == 'dispatch' else r['kind']}"
                              for k, r in enumerate(RECORDS)])
def test_replay_reference_call(dev, i):
    r = RECORDS[i]
    dev.clear_error()
    if r["kind"] == "dispatch":
        _replay_dispatch(dev, i, r)
    else:
        _replay_batch(dev, i, r)
