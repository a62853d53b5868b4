"""The golden trace (tests/golden/ref_trace.npz) against the CPU oracle.

Every recorded dispatch is re-run through `oracle.shaders.run_shader` from its
recorded inputs, cbuffer bytes and group counts, and must reproduce the
recorded outputs exactly: the fixture and the oracle agree, so a GPU replay
that matches the fixture matches the oracle on the reference's own calls.
With the reference sources present, the fixture is also regenerated and must
be identical to the committed one.
"""
import json
import os

import numpy as np
import pytest

from oracle import shaders

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_trace.npz")


def _records():
    z = np.load(FIXTURE)
    return json.loads(str(z["meta"]))["records"], z


def test_fixture_covers_the_reference_shaders():
    recs, _ = _records()
    names = {r["name"] for r in recs if r["kind"] == "dispatch"}
    kinds = {r["kind"] for r in recs}
    for n in ("add_bias", "bias_relu", "relu", "relu_grad", "relu6", "relu6_grad", "leaky_relu", "leaky_relu_grad",
              "sigmoid", "sigmoid_grad", "add", "scale_add", "grad_accum", "bias_grad", "softmax", "loss",
              "softmax_ce_grad", "argmax_correct", "accumulate_scalar", "rms", "adam", "global_avg_pool",
              "global_avg_pool_backward", "batchnorm_mean_var", "batchnorm_forward", "batchnorm_backward_reduce",
              "batchnorm_backward_dx", "dice_loss", "dice_loss_sums", "dice_loss_grad"):
        assert n in names, n
    assert {"SGDBatch", "SGDBatchClipped"} <= kinds


def test_fixture_matches_oracle():
    recs, z = _records()
    for i, r in enumerate(recs):
        if r["kind"] != "dispatch":
            continue
        ids = {}
        uavs = []
        for j in range(r["nuav"]):
            hid = r["uav_ids"][j]
            a = ids.get(hid) if hid else None
            if a is None:
                a = z[f"r{i}_u{j}_in"].copy()
                if hid:
                    ids[hid] = a
            uavs.append(a)
        srvs = []
        for j in range(r["nsrv"]):
            hid = r["srv_ids"][j]
            srvs.append(ids[hid] if hid in ids else z[f"r{i}_s{j}"].copy())
        shaders.run_shader(r["name"], srvs, uavs, tuple(r["groups"]), bytes.fromhex(r["cb"]))
        for j in range(r["nuav"]):
            want = z[f"r{i}_u{j}_out"]
            assert np.array_equal(uavs[j].view(np.uint32), want.view(np.uint32)) or \
                np.allclose(uavs[j], want, equal_nan=True, rtol=0, atol=0), (i, r["name"], j)


@pytest.mark.reference
def test_fixture_regenerates_identically(reference_dir, tmp_path, monkeypatch):
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "make_golden", os.path.join(os.path.dirname(FIXTURE), "make_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = tmp_path / "trace.npz"
    monkeypatch.setattr(mod, "OUT", str(out))
    mod.main(reference_dir)
    a, b = np.load(FIXTURE), np.load(out)
    assert sorted(a.files) == sorted(b.files)
    for k in a.files:
        if k == "meta":
            assert json.loads(str(a[k]))["records"] == json.loads(str(b[k]))["records"]
        else:
            assert np.array_equal(a[k].view(np.uint32), b[k].view(np.uint32)), k
