"""Make tests/golden/ref_trace.npz from the reference's own Python.

    python tests/golden/make_golden.py [REFERENCE_DIR]

The unmodified reference `nn_engine.py` is imported over a recording `FakeLib`
(the NumPy restatement of its native engine, `oracle/fakelib.py`).  It then runs
its own Functions, autograd, optimizers, Metrics and ComputeGraph on small
seeded inputs.  Every engine call that changes device state is recorded with
the buffers it touches, before and after:

* a dispatch (RunShader / RunShaderAlloc / RunSequence commands): the shader
  name, the reference's own cbuffer bytes and group counts, the SRV contents,
  and the UAV contents before and after;
* SGDBatch / SGDBatchClipped: the parameter and gradient arrays, the
  reference's lr / clip / max-norm arguments, and the parameters after.

What the reference contributes: the inputs, which shader runs with which
cbuffer words, group counts and buffer sizes (its packing code), and the
scalar math it does in Python (Adam's bias-corrected step size, clip values).
The "after" contents come from the oracle, which was pinned to the reference's
own checks (tests/test_oracle_pinned.py).  `tests/test_gpu_golden.py` replays
every record through libdct_cuda.so on a GPU box, where the reference does not
exist.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import fakelib  # noqa: E402

OUT = os.path.join(HERE, "ref_trace.npz")


class Recorder(fakelib.FakeLib):
    def __init__(self):
        super().__init__()
        self.records: list[dict] = []
        self.arrays: dict[str, np.ndarray] = {}
        self._inner = 0          # >0 while inside SGDBatch / SGDBatchClipped (their dispatches are ours)

    def _put(self, key, arr):
        self.arrays[key] = np.array(arr, dtype=np.float32, copy=True)

    def _run(self, name, srv_h, uav_h, groups, cb):
        if self._inner:
            return super()._run(name, srv_h, uav_h, groups, cb)
        i = len(self.records)
        srv = [self._bufs[int(h)].data.copy() if h else np.zeros(0, np.float32) for h in srv_h]
        uav_before = [self._bufs[int(h)].data.copy() if h else np.zeros(0, np.float32) for h in uav_h]
        # aliasing between views (same handle twice) is part of the call
        srv_ids = [int(h) if h else 0 for h in srv_h]
        uav_ids = [int(h) if h else 0 for h in uav_h]
        super()._run(name, srv_h, uav_h, groups, cb)
        for j, a in enumerate(srv):
            self._put(f"r{i}_s{j}", a)
        for j, a in enumerate(uav_before):
            self._put(f"r{i}_u{j}_in", a)
            self._put(f"r{i}_u{j}_out", self._bufs[int(uav_h[j])].data if uav_h[j] else a)
        self.records.append({"kind": "dispatch", "name": name, "groups": [int(g) for g in groups],
                             "cb": bytes(cb).hex(), "nsrv": len(srv), "nuav": len(uav_before),
                             "srv_ids": srv_ids, "uav_ids": uav_ids})

    def _batch(self, kind, params, grads, sizes, n, args, call):
        i = len(self.records)
        n = int(n)
        live = [j for j in range(n) if params[j] and grads[j]]
        for j in live:
            self._put(f"r{i}_p{j}_in", self._bufs[int(params[j])].data)
            self._put(f"r{i}_g{j}", self._bufs[int(grads[j])].data)
        self._inner += 1
        try:
            ret = call()
        finally:
            self._inner -= 1
        for j in live:
            self._put(f"r{i}_p{j}_out", self._bufs[int(params[j])].data)
        self.records.append({"kind": kind, "n": n, "live": live, "sizes": [int(sizes[j]) for j in range(n)],
                             "args": [float(a) for a in args], "ret": None if ret is None else float(ret)})
        return ret

    def _SGDBatch(self, params, grads, sizes, n, lr, clip):
        return self._batch("SGDBatch", params, grads, sizes, n, (lr, clip),
                           lambda: super(Recorder, self)._SGDBatch(params, grads, sizes, n, lr, clip))

    def _SGDBatchClipped(self, params, grads, sizes, n, lr, max_norm):
        return self._batch("SGDBatchClipped", params, grads, sizes, n, (lr, max_norm),
                           lambda: super(Recorder, self)._SGDBatchClipped(params, grads, sizes, n, lr, max_norm))


def workloads(nn, rng):
    T = nn.Tensor
    f32 = np.float32

    # -- dense head: every elementwise Function forward + backward through softmax_ce
    B, K = 16, 24
    x_np = rng.standard_normal((B, K)).astype(f32)
    labels = T(rng.integers(0, K, B).astype(f32))
    for act in (lambda x, b: nn.add_bias(x, b), lambda x, b: nn.bias_relu(x, b),
                lambda x, b: nn.relu(nn.add_bias(x, b)), lambda x, b: nn.relu6(nn.add_bias(x, b)),
                lambda x, b: nn.leaky_relu(nn.add_bias(x, b), 0.2), lambda x, b: nn.sigmoid(nn.add_bias(x, b)),
                lambda x, b: nn.add(nn.bias_relu(x, b), nn.add_bias(x, b))):
        x = T(x_np * f32(4.0), requires_grad=True)
        b = T((0.1 * rng.standard_normal(K)).astype(f32), requires_grad=True)
        loss = nn.softmax_ce(act(x, b), labels)
        loss.backward()
    nn.scale_add(T(x_np), T(x_np[::-1].copy()), 0.5, -2.0)

    # -- dice loss, global average pool, BatchNorm2d, rms
    p = T(rng.random((4, 50)).astype(f32), requires_grad=True)
    t = T((rng.random((4, 50)) > 0.5).astype(f32))
    nn.dice_loss(nn.sigmoid(p), t).backward()
    x4 = T((0.5 + 2 * rng.standard_normal((4, 3, 5, 5))).astype(f32), requires_grad=True)
    bn = nn.BatchNorm2d(3)
    y = bn(x4)
    lab4 = T(rng.integers(0, 3, 4).astype(f32))
    nn.softmax_ce(nn.global_avg_pool2d(y), lab4).backward()
    bn.training = False
    bn(x4)
    nn.rms(T(rng.standard_normal(1000).astype(f32)))

    # -- optimizers
    params = [T(rng.standard_normal(300).astype(f32), requires_grad=True),
              T(rng.standard_normal(37).astype(f32), requires_grad=True)]

    def fake_grads(scale):
        for q in params:
            q.grad = T((scale * rng.standard_normal(q.size)).astype(f32))

    fake_grads(2.0)
    nn.SGD(params, lr=0.05).step(clip=1.0)
    fake_grads(0.01)
    nn.SGD(params, lr=0.05).step(clip=1.0)
    opt = nn.AdamW(params, lr=1e-3, weight_decay=0.01)
    for _ in range(3):
        fake_grads(0.5)
        opt.step(clip=1.0)
    fake_grads(3.0)
    nn.sgd_step_clipped(params, lr=0.1, max_norm=1.0)
    fake_grads(1e-3)
    nn.sgd_step_clipped(params, lr=0.1, max_norm=1.0)

    # -- Metrics
    m = nn.Metrics()
    logits = T((3 * rng.standard_normal((B, K))).astype(f32))
    logits_np = logits.sync().copy()
    lab_m = T(np.argmax(logits_np, axis=1).astype(f32))
    loss = nn.softmax_ce(logits, lab_m)
    m.update(loss, logits, lab_m)
    m.update(loss, logits, labels)
    m.collect(2 * B)

    # -- ComputeGraph: record a forward + backward + SGD, replay it
    w = T((0.1 * rng.standard_normal(K)).astype(f32), requires_grad=True)
    g = nn.ComputeGraph()
    xb = rng.standard_normal((B, K)).astype(f32)
    yb = rng.integers(0, K, B).astype(f32)
    g.trace(lambda X: nn.bias_relu(X, w), nn.SGD([w], lr=0.1), xb, yb, [w], clip=1.0)
    g.replay(rng.standard_normal((B, K)).astype(f32), rng.integers(0, K, B).astype(f32))

    # -- layout ops beside the path: upsample -> concat -> maxpool, forward and backward
    xa = T((2 * rng.standard_normal((2, 3, 6, 8))).astype(f32), requires_grad=True)
    xc = T(rng.standard_normal((2, 2, 12, 16)).astype(f32), requires_grad=True)
    cat = nn.concat([nn.upsample2d(xa, 2, 2), xc])                  # [2, 5, 12, 16]
    pooled = nn.maxpool2d(cat, 2, 2)                                 # [2, 5, 6, 8]
    nn.softmax_ce(nn.global_avg_pool2d(pooled), T(rng.integers(0, 5, 2).astype(f32))).backward()
    xs = T(rng.standard_normal((3, 2, 5, 7)).astype(f32), requires_grad=True)
    up = nn.upsample2d(xs, 3, 2)                                     # uneven scales
    nn.softmax_ce(nn.global_avg_pool2d(nn.maxpool2d(up, 3, 3)), T(rng.integers(0, 2, 3).astype(f32))).backward()
    # forward-only pooling: overlapping windows, ragged edges, and values that never
    # beat the -1e30 start (-inf, NaN, -2e30) -> the 0xFFFFFFFF index
    xp = rng.standard_normal((2, 3, 9, 11)).astype(f32)
    xp[0, 0, :3, :3] = -np.inf
    xp[0, 1, 3:6, 3:6] = np.nan
    xp[1, 2, :2, :] = f32(-2e30)
    nn.maxpool2d(T(xp), 3, 2)
    nn.maxpool2d(T(xp), 2, 3)

    # -- conv output / gradient reshapes, packed as ConvForwardFused and
    #    ConvBackwardFused pack them (engine.cpp:784-792, :816-835)
    lib = nn.lib
    Bc, OC, OH, OW = 2, 5, 3, 4
    P = OH * OW
    mm = T((2 * rng.standard_normal((OC, Bc * P))).astype(f32))
    bias = T(rng.standard_normal(OC).astype(f32))
    fwd = None
    for act in (0, 1, 2):
        out = lib.CreateBuffer(None, Bc * OC * P)
        nn._dispatch(b"conv_reshape", (mm.gpu_buf, bias.gpu_buf), (out,), (Bc * P + 15) // 16, (OC + 15) // 16, 1,
                     u1=Bc, u2=OC, u3=OH, u4=OW, u5=act, cbSize=20)
        if act == 1:
            fwd = out
    dz = T(rng.standard_normal((Bc, OC, OH, OW)).astype(f32))
    for name, srvs in ((b"conv_grad_reshape", (dz.gpu_buf,)), (b"conv_grad_reshape_relu", (dz.gpu_buf, fwd))):
        out = lib.CreateBuffer(None, OC * Bc * P)
        nn._dispatch(name, srvs, (out,), (Bc * P + 15) // 16, (OC + 15) // 16, 1,
                     u1=Bc, u5=OC, u8=OH, u9=OW, cbSize=36)


def main(ref_dir: str):
    rec = Recorder()
    nn = fakelib.load_reference_engine(ref_dir, rec)
    rng = np.random.default_rng(2024)
    workloads(nn, rng)
    meta = json.dumps({"records": rec.records, "source": "reference nn_engine.py over oracle.fakelib.FakeLib"})
    np.savez_compressed(OUT, meta=np.array(meta), **rec.arrays)
    kinds = {}
    for r in rec.records:
        k = r["name"] if r["kind"] == "dispatch" else r["kind"]
        kinds[k] = kinds.get(k, 0) + 1
    print(f"{len(rec.records)} records -> {OUT} ({os.path.getsize(OUT)} bytes)")
    print(json.dumps(kinds, sort_keys=True))


if __name__ == "__main__":
    _repo = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    main(sys.argv[1] if len(sys.argv) > 1 else
         (os.environ.get("DCT_REFERENCE_DIR") or os.path.join(os.path.dirname(_repo), "reference")))
