#!/usr/bin/env python
"""Benchmark of the directcompute_torch hot path on B200 (libdct_cuda.so).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl dct|reference]
                    [--no-per-op] [--no-verify] [--no-strong] [--no-e2e] [--no-cpu]

Metric: achieved HBM GB/s per op, whole job, vs the host-CPU
reference.  The headline workload is BASELINE config C2, the broadcast
elementwise sweep -- one STEP is the 11 ops of C2 on one batch:

  add/sub/mul/div/maximum   A[8192,8192] (op) B[1,8192]          (row broadcast)
  mul/add                   C[64,1,4096] (op) D[1,512,4096]      (outer broadcast)
  exp/log(|x|+1)/tanh/sigmoid on A

Each rank holds the full C2 batch as its shard of a leading-dimension-sharded
global tensor (N x 8192 rows): weak scaling, no collective on this path.
`value` = algorithmic bytes of all ranks / max-over-ranks device time of K
steps (inputs resident in HBM; A is 256 MB, twice L2, and every output is
written fresh, so no step reuses another's lines).  `e2e` is the same metric
through the reference-facing C-ABI with host buffers: per step UpdateBuffer of
the inputs from pinned host memory, the 11 RunShader-level calls, and a
ReadBuffer of every output.

`per_op` adds the other BASELINE configs (C1 latency, C3 reductions, C4 fused
softmax+CE, C5a Adam, C5b BatchNorm) and the layout ops beside the path, each
timed with CUDA events on the library's stream.  Every rank holds the
single-GPU size of each config (weak scaling); at N > 1 the ops whose result
spans shards run through the sharded dct_dist_* entry points.  At N > 1
`strong` times the configs whose global size BASELINE fixes (C3 over 16384
rows, the 2^30 full sum, C4 over 65536 rows, C5a over 1.5e9 elements, C5b over
a batch of 256) split N ways.

After timing, every timed output is read back (whole, or a sample of rows /
planes / blocks where the whole would take long) and compared with the oracle:
bit-exact for the elementwise, broadcast, max / argmax, Adam and the applied
BatchNorm outputs, <= 2 ulp for the transcendentals, <= 4 ulp for softmax
probabilities, rel 1e-5 of float64 accumulation for sums.  At N > 1 the
sharded results are checked against the unsharded oracle: each rank's float64
partials travel through the process group and are folded in rank order.
`parity` reports op -> passed.  The oracle is only the checker here: it runs
after the timed regions and never inside them.

The line ends with compact maps that stay inside a short tail of the output:
`per_op_frac` (op -> fraction of the measured HBM peak), `strong` and `parity`.

`--impl reference` times the reference's CPU path for the same workload: the
NumPy restatement in oracle/ (the reference's own CPU arithmetic for these ops
is NumPy), multithreaded over row chunks on this host's cores, on a bounded
sample of the batch.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "achieved HBM GB/s (% of 8 TB/s) per op at 1/2/4/8 B200 vs host-CPU ref"
NOMINAL_HBM_GBS = 8000.0

# C2 shapes
A_ROWS, A_COLS = 8192, 8192
OC_P, OC_R, OC_Q = 64, 512, 4096
ROWBCAST_BYTES = 4 * (2 * A_ROWS * A_COLS + A_COLS)
OUTER_BYTES = 4 * (OC_P * OC_R * OC_Q + OC_P * OC_Q + OC_R * OC_Q)
UNARY_BYTES = 4 * 2 * A_ROWS * A_COLS
C2_BINARY = ("add", "sub", "mul", "div", "maximum")
C2_OUTER = ("mul", "add")
C2_UNARY = ("exp", "log_abs1p", "tanh", "sigmoid")

# dram__bytes_read.sum + dram__bytes_write.sum of one full-size launch, from the
# ncu capture summarised in profiles/k_rowvec_chunk_c2_rowbcast_add.md (the
# bench's own workload: 512 MB on the device, one launch captured)
NCU_TRAFFIC_BYTES = {"c2_rowbcast": 483_056_128}


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------
class Ranks:
    def __init__(self, gpus):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist
            self.torch = torch

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if not self.pg:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def gather(self, a) -> list:
        """Every rank's copy of a same-shaped float64 array, in rank order."""
        a = np.ascontiguousarray(a, dtype=np.float64)
        if not self.pg:
            return [a]
        t = self.torch.from_numpy(a).cuda()
        out = [self.torch.empty_like(t) for _ in range(self.world)]
        self.pg.all_gather(out, t)
        return [o.cpu().numpy() for o in out]

    def all_true(self, flags: list) -> list:
        """Element-wise AND of a list of booleans over the ranks."""
        if not self.pg or not flags:
            return list(flags)
        g = self.gather(np.array([1.0 if f else 0.0 for f in flags]))
        return [bool(min(x[i] for x in g) > 0.5) for i in range(len(flags))]

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# clocks sampled during the timed region (NVML, every 2 ms or as fast as it answers; read-only)
# ---------------------------------------------------------------------------
class Clocks:
    """Samples SM clock, power and clock-event reasons of our GPU while timing."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, pci_bus_id: str, period_s: float = 0.002):
        self.pci = pci_bus_id
        self.period = period_s
        self.rows = []
        self.max_mhz = None
        self._stop = None

    def __enter__(self):
        import threading
        try:
            import pynvml as N
            N.nvmlInit()
            try:
                self.h = N.nvmlDeviceGetHandleByPciBusId(self.pci.encode() if isinstance(self.pci, str) else self.pci)
            except Exception:
                self.h = N.nvmlDeviceGetHandleByIndex(0)
            self.N = N
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
            # one untimed round of the queries the sampler makes: the first calls are slow
            # and would otherwise eat a short timed region
            N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM)
            N.nvmlDeviceGetPowerUsage(self.h)
            (getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or
             N.nvmlDeviceGetCurrentClocksThrottleReasons)(self.h)
        except Exception as e:                      # no NVML: record why
            self.err = repr(e)
            return self
        self._stop = threading.Event()

        def loop():
            N, h = self.N, self.h
            get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                N.nvmlDeviceGetCurrentClocksThrottleReasons
            k, watts = 0, None
            while not self._stop.is_set():
                try:
                    if k % 8 == 0:                  # the power query is the slow one: every 8th sample
                        watts = N.nvmlDeviceGetPowerUsage(h) / 1000.0
                    self.rows.append((N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM), watts, int(get_reasons(h)),
                                      time.monotonic()))
                except Exception:
                    pass
                k += 1
                self._stop.wait(self.period)
        self._t = threading.Thread(target=loop, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        if self._stop is not None:
            self._stop.set()
            self._t.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0,
                    "source": "nvml", "note": getattr(self, "err", "timed region shorter than one sample")}
        reasons = sorted({name for _, _, r, _ in self.rows for bit, name in self.REASONS.items() if r & bit})
        sm = [r[0] for r in self.rows]
        watts = [r[1] for r in self.rows if r[1] is not None]
        span = self.rows[-1][3] - self.rows[0][3]
        period = span / (len(self.rows) - 1) * 1e3 if len(self.rows) > 1 else None
        return {"sm_mhz": float(np.median(sm)), "sm_min_mhz": float(min(sm)), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.rows),
                "power_w_max": round(max(watts), 1) if watts else None,
                "source": "nvml", "period_ms": round(period, 2) if period else None}


# ---------------------------------------------------------------------------
# device side
# ---------------------------------------------------------------------------
class Lib:
    def __init__(self):
        import ctypes
        from directcompute_torch_b200 import load_library
        from directcompute_torch_b200._abi import BINARY, REDUCE, UNARY, check
        self.C = ctypes
        self.lib = load_library()
        if not self.lib.InitEngine():
            raise RuntimeError("InitEngine failed: " + self.lib.dct_last_error().decode())
        self.BINARY, self.REDUCE, self.UNARY, self._check = BINARY, REDUCE, UNARY, check
        self.launches = 0

    def check(self, rc, what):
        self._check(self.lib, rc, what)

    def new(self, n):
        h = self.lib.dct_create_buffer(int(n))
        if not h:
            raise RuntimeError("allocation failed: " + self.lib.dct_last_error().decode())
        return h

    def read(self, h, offset, count, dtype=np.float32):
        """`count` elements of buffer `h` from element `offset` (a blocking copy)."""
        out = np.empty(int(count), np.float32)
        self.check(self.lib.dct_copy_d2h(h, out.ctypes.data, int(offset), int(count)), "read")
        return out.view(dtype)

    def fill(self, h, seed, offset, dist, a, b):
        self.check(self.lib.dct_fill_random(h, seed, offset, dist, a, b), "fill")

    def shape(self, s):
        return (self.C.c_int64 * len(s))(*s)

    def binary(self, op, a, sa, b, sb, out):
        self.check(self.lib.dct_binary(self.BINARY[op], a, sa, len(sa), b, sb, len(sb), out), "binary")
        self.launches += 1

    def unary(self, op, x, y, n):
        self.check(self.lib.dct_unary(self.UNARY[op], x, y, n, 0.0), "unary")
        self.launches += 1

    def run(self, name, srvs, uavs, groups, words):
        """RunShader by reference shader name with the cbuffer `words` (u32)."""
        C = self.C
        sv = (C.c_void_p * max(1, len(srvs)))(*srvs)
        uv = (C.c_void_p * max(1, len(uavs)))(*uavs)
        th = (C.c_uint * 3)(*groups)
        cb = (C.c_uint * max(1, len(words)))(*words)
        self.lib.RunShader(name.encode(), sv, len(srvs), uv, len(uavs), th, C.cast(cb, C.c_void_p), 4 * len(words))

    def time(self, fn, iters):
        self.lib.dct_timer_start()
        for _ in range(iters):
            fn()
        ms = self.lib.dct_timer_stop_ms()
        if ms < 0:
            raise RuntimeError("timer failed: " + self.lib.dct_last_error().decode())
        return ms


class C2:
    """The headline workload: BASELINE config C2 (seed 1), resident in HBM."""

    def __init__(self, L: Lib, rank: int, only: str | None = None):
        self.L = L
        n = A_ROWS * A_COLS
        self.A = L.new(n)
        self.B = L.new(A_COLS)
        self.Cc = L.new(OC_P * OC_Q)
        self.D = L.new(OC_R * OC_Q)
        seed = 1 + 1000 * rank
        L.fill(self.A, seed, 0, 1, 0.0, 1.0)
        L.fill(self.B, seed, 1, 0, 0.5, 2.0)
        L.fill(self.Cc, seed, 2, 1, 0.0, 1.0)
        L.fill(self.D, seed, 3, 1, 0.0, 1.0)
        want = (lambda k: only is None or only == k)
        self.out_b = {op: L.new(n) for op in C2_BINARY if want(f"c2_rowbcast_{op}")}
        self.out_o = {op: L.new(OC_P * OC_R * OC_Q) for op in C2_OUTER if want(f"c2_outer_{op}")}
        self.out_u = {op: L.new(n) for op in C2_UNARY if want(f"c2_unary_{op}")}
        self.sA = L.shape([A_ROWS, A_COLS])
        self.sB = L.shape([1, A_COLS])
        self.sC = L.shape([OC_P, 1, OC_Q])
        self.sD = L.shape([1, OC_R, OC_Q])
        self.ops = []
        for op in self.out_b:
            self.ops.append((f"c2_rowbcast_{op}", ROWBCAST_BYTES,
                             lambda op=op: L.binary(op, self.A, self.sA, self.B, self.sB, self.out_b[op])))
        for op in self.out_o:
            self.ops.append((f"c2_outer_{op}", OUTER_BYTES,
                             lambda op=op: L.binary(op, self.Cc, self.sC, self.D, self.sD, self.out_o[op])))
        for op in self.out_u:
            self.ops.append((f"c2_unary_{op}", UNARY_BYTES, lambda op=op: L.unary(op, self.A, self.out_u[op], n)))
        if not self.ops:
            raise SystemExit(f"--only {only}: no such C2 op")
        self.step_bytes = sum(b for _, b, _ in self.ops)
        self.launches_per_step = len(self.ops)

    def step(self):
        for _, _, fn in self.ops:
            fn()


def run_e2e(L: Lib, c2: C2, steps: int, warmup: int):
    """Same C2 step through the reference-facing C-ABI with pinned host buffers."""
    C = L.C
    lib = L.lib
    n = A_ROWS * A_COLS
    hostA = lib.dct_host_alloc(4 * n)
    hostB = lib.dct_host_alloc(4 * A_COLS)
    hostC = lib.dct_host_alloc(4 * OC_P * OC_Q)
    hostD = lib.dct_host_alloc(4 * OC_R * OC_Q)
    hostOut = lib.dct_host_alloc(4 * OC_P * OC_R * OC_Q)
    if not all((hostA, hostB, hostC, hostD, hostOut)):
        raise RuntimeError("pinned allocation failed")
    for h, src, cnt in ((hostA, c2.A, n), (hostB, c2.B, A_COLS), (hostC, c2.Cc, OC_P * OC_Q), (hostD, c2.D, OC_R * OC_Q)):
        L.check(lib.dct_copy_d2h(src, h, 0, cnt), "e2e setup")
    fp = C.POINTER(C.c_float)
    outs = [c2.out_b[o] for o in C2_BINARY] + [c2.out_o[o] for o in C2_OUTER] + [c2.out_u[o] for o in C2_UNARY]

    def step():
        lib.UpdateBuffer(c2.A, C.cast(hostA, fp))
        lib.UpdateBuffer(c2.B, C.cast(hostB, fp))
        lib.UpdateBuffer(c2.Cc, C.cast(hostC, fp))
        lib.UpdateBuffer(c2.D, C.cast(hostD, fp))
        c2.step()
        for o in outs:
            lib.ReadBuffer(o, C.cast(hostOut, fp))

    for _ in range(warmup):
        step()
    lib.dct_synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    lib.dct_synchronize()
    dt = time.perf_counter() - t0
    h2d = 4 * (n + A_COLS + OC_P * OC_Q + OC_R * OC_Q)
    d2h = 4 * (len(C2_BINARY) * n + len(C2_OUTER) * OC_P * OC_R * OC_Q + len(C2_UNARY) * n)
    for h in (hostA, hostB, hostC, hostD, hostOut):
        lib.dct_host_free(h)
    err = lib.dct_error_code()
    if err:
        raise RuntimeError("e2e: " + lib.dct_last_error().decode())
    return dt, h2d, d2h


def link_bandwidth(L: Lib, nbytes: int = 1 << 29, reps: int = 3):
    """Pinned host<->device copy rates (GB/s) on the library's stream: the
    ceiling for the e2e step's copies."""
    lib = L.lib
    n = nbytes // 4
    h = L.new(n)
    host = lib.dct_host_alloc(nbytes)
    if not host:
        raise RuntimeError("pinned allocation failed")
    L.check(lib.dct_copy_h2d(h, host, 0, n), "link h2d")
    lib.dct_synchronize()
    lib.dct_timer_start()
    for _ in range(reps):
        L.check(lib.dct_copy_h2d(h, host, 0, n), "link h2d")
    h2d = nbytes * reps / (lib.dct_timer_stop_ms() * 1e-3) / 1e9
    lib.dct_timer_start()
    for _ in range(reps):
        L.check(lib.dct_copy_d2h(h, host, 0, n), "link d2h")
    d2h = nbytes * reps / (lib.dct_timer_stop_ms() * 1e-3) / 1e9
    lib.dct_host_free(host)
    lib.ReleaseBuffer(h)
    return h2d, d2h


# ---------------------------------------------------------------------------
# parity of what was timed (the oracle as the checker, after the timed regions)
# ---------------------------------------------------------------------------
class Parity:
    """op -> passed, from checks run after the op was timed.

    A check computes its local figures, takes every collective it needs before
    it asserts anything (so all ranks run the same collective steps whatever
    fails), then asserts.  `finish()` ANDs each result over the ranks."""

    def __init__(self, enabled: bool):
        self.enabled = enabled
        self.res = {}
        self.msg = {}

    def run(self, name: str, fn) -> None:
        if not self.enabled:
            return
        try:
            fn()
            self.res[name] = True
        except AssertionError as e:
            self.res[name] = False
            self.msg[name] = str(e)[:200]

    def finish(self, ranks: "Ranks") -> dict:
        names = list(self.res)
        ok = ranks.all_true([self.res[n] for n in names])
        return dict(zip(names, ok))


def _bits_equal(got, want) -> bool:
    g = np.ascontiguousarray(got, np.float32).ravel()
    w = np.ascontiguousarray(want, np.float32).ravel()
    return g.size == w.size and bool(np.all((g.view(np.uint32) == w.view(np.uint32)) | (np.isnan(g) & np.isnan(w))))


def _assert_bits(got, want, what):
    if not _bits_equal(got, want):
        g = np.ascontiguousarray(got, np.float32).ravel()
        w = np.ascontiguousarray(want, np.float32).ravel()
        if g.size != w.size:
            raise AssertionError(f"{what}: {g.size} values, expected {w.size}")
        bad = np.flatnonzero(g.view(np.uint32) != w.view(np.uint32))[:3]
        raise AssertionError(f"{what}: not bit-exact at {bad.tolist()}: {g[bad].tolist()} vs {w[bad].tolist()}")


def _assert_rel(got, want64, tol, what, atol=0.0):
    got = np.asarray(got, np.float64)
    want64 = np.asarray(want64, np.float64)
    err = np.abs(got - want64)
    if not np.all(err <= tol * np.abs(want64) + atol):
        i = int(np.argmax(err - tol * np.abs(want64)))
        raise AssertionError(f"{what}: {got.ravel()[i]} vs {want64.ravel()[i]} beyond rel {tol}")


def verify_c2(L: "Lib", c2: "C2", parity: Parity):
    """Sampled rows of every C2 output of the last step against NumPy float32 (bit-exact)
    and the float64-rounded transcendentals (<= 2 ulp)."""
    if not parity.enabled:
        return
    from oracle import newops as O
    rows = np.unique(np.linspace(0, A_ROWS - 1, 64).astype(np.int64))
    A = np.stack([L.read(c2.A, r * A_COLS, A_COLS) for r in rows])
    B = L.read(c2.B, 0, A_COLS).reshape(1, A_COLS)
    for op, h in c2.out_b.items():
        def chk(op=op, h=h):
            got = np.stack([L.read(h, r * A_COLS, A_COLS) for r in rows])
            _assert_bits(got, O.binary(op, A, B), op)
        parity.run(f"c2_rowbcast_{op}", chk)
    if c2.out_o:
        Cc = L.read(c2.Cc, 0, OC_P * OC_Q).reshape(OC_P, OC_Q)
        D = L.read(c2.D, 0, OC_R * OC_Q).reshape(OC_R, OC_Q)
        pairs = [(p, r) for p in np.linspace(0, OC_P - 1, 8).astype(int)
                 for r in np.linspace(0, OC_R - 1, 16).astype(int)]
        for op, h in c2.out_o.items():
            def chk(op=op, h=h):
                got = np.stack([L.read(h, (p * OC_R + r) * OC_Q, OC_Q) for p, r in pairs])
                want = np.stack([O.binary(op, Cc[p], D[r]) for p, r in pairs])
                _assert_bits(got, want, op)
            parity.run(f"c2_outer_{op}", chk)
    for op, h in c2.out_u.items():
        def chk(op=op, h=h):
            got = np.stack([L.read(h, r * A_COLS, A_COLS) for r in rows])
            want = O.unary_f64(op, A)
            nan = np.isnan(want)
            assert np.array_equal(np.isnan(got), nan), f"{op}: NaN pattern"
            u = int(O.ulp_diff(got[~nan], want[~nan]).max())
            assert u <= 2, f"{op}: {u} ulp"
        parity.run(f"c2_unary_{op}", chk)


# ---------------------------------------------------------------------------
# per-op breakdown of the other BASELINE configs
# ---------------------------------------------------------------------------
PER_OP_SECTIONS = {"c1": ("c1_dense_step_eager", "c1_dense_step_graph"),
                   "c3": ("c3_sum_axis-1", "c3_sum_axis0", "c3_mean_axis-1", "c3_mean_axis0", "c3_max_axis-1",
                          "c3_max_axis0", "c3_argmax_axis-1", "c3_argmax_axis0"),
                   "c3f": ("c3_fullsum_2^30", "c3_fullsum_2^28_small"), "c4": ("c4_softmax_ce_fused",),
                   "c5a": ("c5a_adam_1.5e9", "c5a_adam_1.5e8_small"),
                   "c5b": ("c5b_batchnorm_fwd", "c5b_batchnorm_bwd"),
                   "layout": ("f3_upsample2x_fwd", "f3_upsample2x_bwd", "f3_concat", "f3_slice", "f3_maxpool2x2_fwd",
                              "f3_maxpool2x2_fused_fwd_bwd", "f4_conv_reshape_relu", "f4_conv_grad_reshape_relu"),
                   "dice": ("f1_dice_sums", "f1_dice_loss", "f1_dice_grad")}
#: the configs whose global size BASELINE fixes, timed split N ways at N > 1
STRONG_SECTIONS = ("c3", "c3f", "c4", "c5a", "c5b")


def _oracle_shaders():
    from oracle import shaders
    return shaders


class Suite:
    """One pass over the per-op configs.

    split "weak": every rank holds the single-GPU size of each config.
    split "strong": every rank holds 1/N of it (C3 16384/N rows, the full sum
    2^30/N elements, C4 65536/N rows, C5a 1.5e9/N elements, C5b 256/N samples).
    With a communicator (N > 1) the ops whose result spans shards -- axis-0
    and full reductions, the softmax-CE loss, BatchNorm statistics -- run
    through the sharded dct_dist_* entry points: one exchange of small per-rank
    records each, over NVLink peer memory or the NCCL all-gather fallback."""

    def __init__(self, L: "Lib", ranks, comm=None, split: str = "weak", parity: Parity | None = None,
                 iters: int = 10, warmup: int = 3, only: str | None = None):
        self.L, self.lib, self.C = L, L.lib, L.C
        self.ranks, self.rank, self.world, self.comm = ranks, ranks.rank, ranks.world, comm
        self.div = ranks.world if split == "strong" else 1
        self.parity = parity if parity is not None else Parity(False)
        self.iters, self.warmup, self.only = iters, warmup, only
        self.res = {}

    def want(self, key):
        return self.only is None or self.only in PER_OP_SECTIONS[key]

    def measure(self, name, nbytes, fn, launches, it=None):
        if self.only is not None and name != self.only:
            return False
        it = it or self.iters
        for _ in range(self.warmup):
            fn()
        ms = self.L.time(fn, it) / it
        self.res[name] = {"gbs": round(nbytes / (ms * 1e-3) / 1e9, 1), "ms": round(ms, 4), "bytes": int(nbytes),
                          "launches": launches}
        return True

    def check(self, name, fn):
        if name in self.res:
            self.parity.run(name, fn)

    def run(self, sections=None):
        sections = sections or tuple(PER_OP_SECTIONS)
        for key, fn in (("c1", self._c1), ("c3", self._c3), ("c3f", self._c3f), ("c4", self._c4),
                        ("c5a", self._c5a), ("c5b", self._c5b), ("layout", self._layout),
                        ("dice", self._dice)):
            if key in sections and self.want(key):
                fn()
        self.lib.DrainPool()
        return self.res

    # -- C1 -----------------------------------------------------------------------------
    def _c1(self):
        """C1 (latency, not bandwidth): X[256,784], b[784]; fwd bias_relu, column sums, full sum;
        bwd relu_grad, bias_grad (+ a grad accumulation), as reference RunShader calls one by one
        (eager) and as one RunSequence of the same commands (replayed as a CUDA graph)."""
        L, C, lib = self.L, self.C, self.lib
        from directcompute_torch_b200._abi import SeqCmd
        M, N = 256, 784
        h = {k: L.new(n) for k, n in (("x", M * N), ("b", N), ("y", M * N), ("col", N), ("tot", 1), ("ones", M * N),
                                      ("dx", M * N), ("db", N), ("acc", N))}
        L.fill(h["x"], 0 + 1000 * self.rank, 0, 1, 0.0, 1.0)
        L.fill(h["b"], 0 + 1000 * self.rank, 1, 0, -0.1, 0.1)
        lib.ClearBuffer(h["acc"])
        ones = np.ones(M * N, np.float32)
        L.check(lib.dct_copy_h2d(h["ones"], ones.ctypes.data, 0, M * N), "ones")
        g = ((M * N + 255) // 256, 1, 1)
        spec = [("bias_relu", ["x", "b"], ["y"], g, [M, N]), ("bias_grad", ["y"], ["col"], (N, 1, 1), [M, N, N, 1]),
                ("dct_reduce_all", ["y"], ["tot"], (1, 1, 1), [0, M * N]),
                ("relu_grad", ["ones", "y"], ["dx"], g, [M * N]),
                ("bias_grad", ["dx"], ["db"], (N, 1, 1), [M, N, N, 1]),
                ("grad_accum", ["db"], ["acc"], ((N + 255) // 256, 1, 1), [N])]
        for name in ("bias_relu", "bias_grad", "relu_grad", "grad_accum"):
            lib.CompileShader(name.encode(), "")
        calls, cmds = [], []
        for name, srv, uav, grp, words in spec:
            sv = (C.c_void_p * 8)(*[h[k] for k in srv])
            uv = (C.c_void_p * 4)(*[h[k] for k in uav])
            th = (C.c_uint * 3)(*grp)
            cb = np.array(words, np.uint32)
            calls.append((name.encode(), sv, len(srv), uv, len(uav), th, cb, 4 * len(words)))
            c = SeqCmd()
            c.shader = lib.ResolveShader(name.encode())
            for i, k in enumerate(srv):
                c.srvs[i] = h[k]
            for i, k in enumerate(uav):
                c.uavs[i] = h[k]
            c.srvCount, c.uavCount = len(srv), len(uav)
            c.threads[0], c.threads[1], c.threads[2] = grp
            C.memmove(c.cbData, cb.ctypes.data, 4 * len(words))
            c.cbSize = 4 * len(words)
            cmds.append(c)
        arr = (SeqCmd * len(cmds))(*cmds)
        steps = [0]

        def eager():
            steps[0] += 1
            for name, sv, ns, uv, nu, th, cb, nb in calls:
                lib.RunShader(name, sv, ns, uv, nu, th, cb.ctypes.data, nb)

        def graph():
            steps[0] += 1
            lib.RunSequence(C.cast(arr, C.c_void_p), len(cmds))
        # C1 forward + backward algorithmic bytes
        nbytes = 4 * (3 * M * N + 2 * N + 1) + 4 * (3 * M * N + N)
        # kernels per step: bias_relu and grad_accum one each; each column sum (bias_grad)
        # and the full sum two (partials, then their fold); relu_grad one eager, while
        # the graph runs bias_relu + bias_grad and relu_grad + bias_grad + grad_accum
        # each as one pass (+ its fold), and the full sum as two
        self.measure("c1_dense_step_eager", nbytes, eager, 9, it=200)
        self.measure("c1_dense_step_graph", nbytes, graph, 6, it=200)
        for k in ("c1_dense_step_eager", "c1_dense_step_graph"):
            if k in self.res:
                self.res[k]["us_per_step"] = round(self.res[k]["ms"] * 1e3, 2)

        def chk():
            S = _oracle_shaders()
            x, b = L.read(h["x"], 0, M * N), L.read(h["b"], 0, N)
            y = S.bias_relu(x, b, M, N)
            _assert_bits(L.read(h["y"], 0, M * N), y, "bias_relu")
            y64 = y.astype(np.float64).reshape(M, N)
            _assert_rel(L.read(h["col"], 0, N), y64.sum(0), 1e-5, "bias_grad(y)", atol=1e-30)
            _assert_rel(L.read(h["tot"], 0, 1), [y64.sum()], 1e-5, "sum(y)")
            dx = S.relu_grad(ones, y, M * N)
            _assert_bits(L.read(h["dx"], 0, M * N), dx, "relu_grad")
            db = L.read(h["db"], 0, N)
            _assert_rel(db, dx.astype(np.float64).reshape(M, N).sum(0), 1e-5, "bias_grad(dx)", atol=1e-30)
            acc = np.zeros(N, np.float32)
            for _ in range(steps[0]):
                acc = S.grad_accum(acc, db, N)
            _assert_bits(L.read(h["acc"], 0, N), acc, f"grad_accum x{steps[0]}")
        self.check("c1_dense_step_eager", chk)
        self.check("c1_dense_step_graph", chk)
        for v in h.values():
            lib.ReleaseBuffer(v)

    # -- C3 -----------------------------------------------------------------------------
    def _c3(self):
        """R[16384,4096] ~ N(0,1) + 0.1% +-1e4 outliers (seed 2); axis -1 and axis 0 reductions."""
        L, C, lib, comm = self.L, self.C, self.lib, self.comm
        rows, cols = 16384 // self.div, 4096
        R = L.new(rows * cols)
        out = L.new(max(rows, cols))
        L.fill(R, 2 + 1000 * self.rank, 0, 1, 0.0, 1.0)
        rng = np.random.default_rng(2 + 1000 * self.rank)
        k = (rows * cols) // 1000
        idx = rng.choice(rows * cols, k, replace=False).astype(np.int64)
        vals = np.where(rng.integers(0, 2, k) == 1, 1e4, -1e4).astype(np.float32)
        L.check(lib.dct_scatter(R, idx.ctypes.data_as(C.POINTER(C.c_int64)),
                                vals.ctypes.data_as(C.POINTER(C.c_float)), k), "scatter")
        rbytes = 4 * rows * cols
        total = rows * self.world
        if self.parity.enabled:
            Rh = L.read(R, 0, rows * cols).reshape(rows, cols)
            srow = np.unique(np.linspace(0, rows - 1, 256).astype(np.int64))
            # this rank's float64 column partials and (max, global first index); every rank's, in rank order
            colsum = self.ranks.gather(Rh.astype(np.float64).sum(0))
            cmax = self.ranks.gather(Rh.max(0).astype(np.float64))
            carg = self.ranks.gather((Rh.argmax(0) + rows * self.rank).astype(np.float64))
            gsum = np.zeros(cols)
            for p in colsum:
                gsum += p
            gmax, garg = cmax[0].copy(), carg[0].copy()
            for m_, a_ in zip(cmax[1:], carg[1:]):
                better = m_ > gmax                    # strict: an earlier rank keeps a tie (first index)
                gmax = np.where(better, m_, gmax)
                garg = np.where(better, a_, garg)
        for op in ("sum", "mean", "max", "argmax"):
            if self.measure(f"c3_{op}_axis-1", rbytes + 4 * rows,
                            lambda op=op: L.check(lib.dct_reduce(L.REDUCE[op], R, rows, cols, 1, out, None), op), 1):
                def chk(op=op):
                    got = L.read(out, 0, rows, np.int32 if op == "argmax" else np.float32)[srow]
                    sub = Rh[srow]
                    if op in ("sum", "mean"):
                        want = sub.astype(np.float64).sum(1) / (cols if op == "mean" else 1)
                        _assert_rel(got, want, 1e-5, f"{op} axis -1")
                    elif op == "max":
                        _assert_bits(got, sub.max(1), "max axis -1")
                    else:
                        assert np.array_equal(got, sub.argmax(1)), "argmax axis -1"
                self.check(f"c3_{op}_axis-1", chk)
            if comm is None:
                fn = (lambda op=op: L.check(lib.dct_reduce(L.REDUCE[op], R, 1, rows, cols, out, None), op))
                nl = 2
            else:                      # rows of a [rows * world, cols] matrix, reduced over all of them
                fn = (lambda op=op: comm.reduce(op, R, 1, rows, cols, rows * self.rank, total, out))
                nl = 5
            if self.measure(f"c3_{op}_axis0", rbytes + 4 * cols, fn, nl):
                def chk(op=op):
                    got = L.read(out, 0, cols, np.int32 if op == "argmax" else np.float32)
                    if op in ("sum", "mean"):
                        _assert_rel(got, gsum / (total if op == "mean" else 1), 1e-5, f"{op} axis 0")
                    elif op == "max":
                        _assert_bits(got, gmax.astype(np.float32), "max axis 0")
                    else:
                        assert np.array_equal(got, garg.astype(np.int32)), "argmax axis 0"
                self.check(f"c3_{op}_axis0", chk)
        lib.ReleaseBuffer(R)
        lib.ReleaseBuffer(out)

    def _c3f(self):
        """The full sum of a flat U(-1,1) vector of 2^30 elements (2^28: the small profiling case)."""
        L, lib, comm = self.L, self.lib, self.comm
        small = self.only == "c3_fullsum_2^28_small"
        nv = (1 << (28 if small else 30)) // self.div
        name = "c3_fullsum_2^28_small" if small else "c3_fullsum_2^30"
        V = L.new(nv)
        out = L.new(1)
        L.fill(V, 2 + 1000 * self.rank, 7, 0, -1.0, 1.0)
        if comm is None:
            fs = lambda: L.check(lib.dct_reduce_all(0, V, nv, out, None), "fullsum")  # noqa: E731
        else:
            fs = lambda: comm.reduce_all("sum", V, nv, out)  # noqa: E731
        if self.measure(name, 4 * nv, fs, 2 if comm is None else 5, it=5) and self.parity.enabled:
            acc = 0.0
            step = 1 << 26
            for s in range(0, nv, step):
                acc += float(L.read(V, s, min(step, nv - s)).astype(np.float64).sum())
            want = sum(float(p[0]) for p in self.ranks.gather(np.array([acc])))
            self.check(name, lambda: _assert_rel(L.read(out, 0, 1), [want], 1e-5, "full sum"))
        lib.ReleaseBuffer(V)
        lib.ReleaseBuffer(out)

    # -- C4 -----------------------------------------------------------------------------
    def _c4(self):
        """C4: fused softmax + CE fwd+bwd on [65536,1000] (per rank, or split N ways), int labels (seed 3)."""
        L, lib, comm = self.L, self.lib, self.comm
        B, K = 65536 // self.div, 1000
        gB = B * self.world
        X = L.new(B * K)
        L.fill(X, 3 + 1000 * self.rank, 0, 1, 0.0, 3.0)
        lab = np.random.default_rng(3 + 1000 * self.rank).integers(0, K, B).astype(np.int32)
        Lb = L.new(B)
        L.check(lib.dct_copy_h2d(Lb, lab.ctypes.data, 0, B), "labels")
        P, G, LS = L.new(B * K), L.new(B * K), L.new(1)
        if comm is None:
            fn = lambda: L.check(lib.dct_softmax_ce(X, Lb, 1, B, K, P, G, LS, None, float(B), float(B)), "smce")  # noqa
            nl = 2
        else:
            fn = lambda: comm.softmax_ce(X, Lb, B, K, probs=P, dlogits=G, loss=LS, global_rows=gB,  # noqa: E731
                                         labels_int32=True)
            nl = 6
        if self.measure("c4_softmax_ce_fused", 4 * (3 * B * K + B) + 4, fn, nl) and self.parity.enabled:
            from oracle import newops as O
            loss = 0.0
            step = 4096
            for s in range(0, B, step):
                n = min(step, B - s)
                _, rl, _ = O.softmax_ce_rows_f64(L.read(X, s * K, n * K).reshape(n, K), lab[s:s + n])
                loss += float(rl.sum())
            want = sum(float(p[0]) for p in self.ranks.gather(np.array([loss]))) / gB

            def chk():
                rows = np.unique(np.linspace(0, B - 1, 256).astype(np.int64))
                x = np.stack([L.read(X, r * K, K) for r in rows])
                p_ref, _, _ = O.softmax_ce_rows_f64(x, lab[rows])
                p = np.stack([L.read(P, r * K, K) for r in rows])
                u = int(O.ulp_diff(p, p_ref).max())
                assert u <= 4, f"probs {u} ulp"
                _assert_bits(np.stack([L.read(G, r * K, K) for r in rows]),
                             O.softmax_ce_dlogits(p, lab[rows], gB), "dlogits")
                _assert_rel(L.read(LS, 0, 1), [want], 1e-5, "mean CE loss")
            self.check("c4_softmax_ce_fused", chk)
        for h in (X, Lb, P, G, LS):
            lib.ReleaseBuffer(h)

    # -- C5a ----------------------------------------------------------------------------
    def _c5a(self):
        """C5a: Adam on 1.5e9 fp32 (per rank, or split N ways; seed 4), zero m/v.  The small case
        (1.5e8, 2.4 GB held, run only when named) is for profiler captures of the same kernel."""
        L, lib = self.L, self.lib
        small = self.only == "c5a_adam_1.5e8_small"
        n = (150_000_000 if small else 1_500_000_000) // self.div
        W, Gr, M, Vv = L.new(n), L.new(n), L.new(n), L.new(n)
        L.fill(W, 4 + 1000 * self.rank, 0, 1, 0.0, 0.02)
        L.fill(Gr, 4 + 1000 * self.rank, 1, 1, 0.0, 1e-3)
        lib.ClearBuffer(M)
        lib.ClearBuffer(Vv)
        blk = 4096
        offs = np.linspace(0, n - blk, 64).astype(np.int64).tolist()
        if self.parity.enabled:                      # sampled blocks of the initial state
            w0 = np.concatenate([L.read(W, o, blk) for o in offs])
            g0 = np.concatenate([L.read(Gr, o, blk) for o in offs])
        t = [0]

        def adam():
            t[0] += 1
            step = 1e-3 * (1 - 0.999 ** t[0]) ** 0.5 / (1 - 0.9 ** t[0])
            L.check(lib.dct_adam(W, M, Vv, Gr, n, step, 0.9, 0.999, 1e-8, 0.0, 1.0), "adam")
        name = "c5a_adam_1.5e8_small" if small else "c5a_adam_1.5e9"
        if self.measure(name, 28 * n, adam, 1, it=10):
            def chk():
                S = _oracle_shaders()
                w, m, v = w0, np.zeros_like(w0), np.zeros_like(w0)
                for k in range(1, t[0] + 1):
                    w, m, v = S.adam(w, m, v, g0, w.size, S.adam_step_size(1e-3, 0.9, 0.999, k), 0.9, 0.999, 1e-8,
                                     0.0, 1.0)
                for h, want, what in ((W, w, "w"), (M, m, "m"), (Vv, v, "v")):
                    _assert_bits(np.concatenate([L.read(h, o, blk) for o in offs]), want, f"adam {what} x{t[0]}")
            self.check(name, chk)
        for h in (W, Gr, M, Vv):
            lib.ReleaseBuffer(h)

    # -- C5b ----------------------------------------------------------------------------
    def _c5b(self):
        """C5b: BatchNorm train fwd / bwd on [256,256,56,56] (per rank, or the batch split N ways; seed 4)."""
        L, lib, comm = self.L, self.lib, self.comm
        N, Cc, S_ = 256 // self.div, 256, 56 * 56
        plane = Cc * S_
        nx = N * plane
        x, dy, y, dx = L.new(nx), L.new(nx), L.new(nx), L.new(nx)
        L.fill(x, 4 + 1000 * self.rank, 10, 1, 0.5, 2.0)
        L.fill(dy, 4 + 1000 * self.rank, 11, 1, 0.0, 1.0)
        gam, bet, rm, rv, bm, bv, dg, db = (L.new(Cc) for _ in range(8))
        for h, v in ((gam, 1.0), (bet, 0.0), (rm, 0.0), (rv, 1.0)):
            arr = np.full(Cc, v, np.float32)
            L.check(lib.dct_copy_h2d(h, arr.ctypes.data, 0, Cc), "bn init")
        lib.dct_synchronize()
        calls = [0]
        eps = 1e-5
        if comm is None:
            def fwd():
                calls[0] += 1
                L.check(lib.dct_batchnorm_forward_train(x, gam, bet, rm, rv, bm, bv, y, N, Cc, S_, eps, 0.1), "bnf")
            bwd = lambda: L.check(lib.dct_batchnorm_backward(x, dy, bm, bv, gam, dg, db, dx, N, Cc, S_, eps),  # noqa
                                  "bnb")
            nf = nb = 4
        else:
            def fwd():
                calls[0] += 1
                comm.batchnorm_forward_train(x, gam, bet, rm, rv, bm, bv, y, N, Cc, S_, eps, 0.1)
            bwd = lambda: comm.batchnorm_backward(x, dy, bm, bv, gam, dg, db, dx, N, Cc, S_, eps)  # noqa: E731
            nf = nb = 7
        gN = N * self.world
        cnt = gN * S_
        samples = sorted({0, N // 2, N - 1})
        if self.measure("c5b_batchnorm_fwd", 4 * 3 * nx, fwd, nf) and self.parity.enabled:
            S = _oracle_shaders()
            s1, s2 = np.zeros(Cc), np.zeros(Cc)
            for i in range(N):
                xi = L.read(x, i * plane, plane).astype(np.float64).reshape(Cc, S_)
                s1 += xi.sum(1)
                s2 += (xi * xi).sum(1)
            g1, g2 = self.ranks.gather(s1), self.ranks.gather(s2)
            t1, t2 = np.zeros(Cc), np.zeros(Cc)
            for a, b in zip(g1, g2):
                t1 += a
                t2 += b
            mean64 = t1 / cnt
            var64 = np.maximum(0.0, t2 / cnt - mean64 * mean64)

            def chk():
                mean, var = L.read(bm, 0, Cc), L.read(bv, 0, Cc)
                _assert_rel(mean, mean64, 1e-6, "batch mean")
                _assert_rel(var, var64, 1e-6, "batch var")
                r_m, r_v = np.zeros(Cc, np.float32), np.ones(Cc, np.float32)
                for _ in range(calls[0]):
                    r_m, r_v = S.batchnorm_running(r_m, r_v, mean64, var64, gN, S_, 0.1)
                _assert_rel(L.read(rm, 0, Cc), r_m, 1e-5, f"running mean x{calls[0]}", atol=1e-7)
                _assert_rel(L.read(rv, 0, Cc), r_v, 1e-5, f"running var x{calls[0]}")
                one, zero = np.ones(Cc, np.float32), np.zeros(Cc, np.float32)
                for i in samples:
                    _assert_bits(L.read(y, i * plane, plane),
                                 S.batchnorm_forward(L.read(x, i * plane, plane), mean, var, one, zero, 1, Cc, S_,
                                                     np.float32(eps)), f"y sample {i}")
            self.check("c5b_batchnorm_fwd", chk)
        if self.measure("c5b_batchnorm_bwd", 4 * 5 * nx, bwd, nb) and self.parity.enabled:
            S = _oracle_shaders()
            mean32, var32 = L.read(bm, 0, Cc), L.read(bv, 0, Cc)
            sx, sd = np.zeros(Cc), np.zeros(Cc)
            for i in range(N):
                xi = L.read(x, i * plane, plane).astype(np.float64).reshape(Cc, S_)
                di = L.read(dy, i * plane, plane).astype(np.float64).reshape(Cc, S_)
                sx += (di * (xi - mean32.astype(np.float64)[:, None])).sum(1)
                sd += di.sum(1)
            gx, gd = self.ranks.gather(sx), self.ranks.gather(sd)
            tx, td = np.zeros(Cc), np.zeros(Cc)
            for a, b in zip(gx, gd):
                tx += a
                td += b
            rstd = (np.float32(1.0) / np.sqrt(var32 + np.float32(eps))).astype(np.float32).astype(np.float64)

            def chk():
                dgam, dbet = L.read(dg, 0, Cc), L.read(db, 0, Cc)
                atol = 1e-6 * np.sqrt(cnt)
                _assert_rel(dgam, tx * rstd, 1e-5, "dgamma", atol=atol)
                _assert_rel(dbet, td, 1e-5, "dbeta", atol=atol)
                one = np.ones(Cc, np.float32)
                for i in samples:
                    want = S.batchnorm_backward_dx(L.read(x, i * plane, plane), L.read(dy, i * plane, plane), mean32,
                                                   var32, one, dgam, dbet, 1, Cc, S_, np.float32(eps), count=cnt)
                    _assert_bits(L.read(dx, i * plane, plane), want, f"dx sample {i}")
            self.check("c5b_batchnorm_bwd", chk)
        for h in (x, dy, y, dx, gam, bet, rm, rv, bm, bv, dg, db):
            lib.ReleaseBuffer(h)

    # -- layout ops ---------------------------------------------------------------------
    def _dice(self):
        """Dice loss beside the path (nn_dice_loss_sums.hlsl:19-55, nn_dice_loss.hlsl:19-53,
        nn_dice_loss_grad.hlsl:17-34; nn_engine.py:1290-1317), dispatched by reference
        shader name with the reference's cbuffer words, on a segmentation batch
        pred / target [64, 1, 512, 512] ~ U(0, 1): 67 MB each, the pair larger than L2.
        No reference config sizes it; the shape is synthetic.  Checks cover the first
        and last sample."""
        L, lib = self.L, self.lib
        for name in ("dice_loss_sums", "dice_loss", "dice_loss_grad"):
            lib.CompileShader(name.encode(), "")
        B, S_ = 64, 512 * 512
        n = B * S_
        seed = 6 + 1000 * self.rank
        p, t, sums, loss, dx = L.new(n), L.new(n), L.new(3 * B), L.new(B), L.new(n)
        L.fill(p, seed, 30, 0, 0.0, 1.0)
        L.fill(t, seed, 31, 0, 0.0, 1.0)
        ends = (0, B - 1)
        g1 = (B, 1, 1)
        if self.measure("f1_dice_sums", 4 * (2 * n + 3 * B), lambda: L.run("dice_loss_sums", [p, t], [sums], g1, [B, S_]), 2):
            def chk_sums():
                got = L.read(sums, 0, 3 * B).reshape(B, 3)
                for b in ends:
                    want = _oracle_shaders().dice_sums(L.read(p, b * S_, S_), L.read(t, b * S_, S_), 1, S_)[0]
                    _assert_rel(got[b], want, 1e-5, f"dice sums sample {b}")
            self.check("f1_dice_sums", chk_sums)
        if self.measure("f1_dice_loss", 4 * (2 * n + B), lambda: L.run("dice_loss", [p, t], [loss], g1, [B, S_]), 2):
            def chk_loss():
                got = L.read(loss, 0, B)
                for b in ends:
                    want = _oracle_shaders().dice_loss(L.read(p, b * S_, S_), L.read(t, b * S_, S_), 1, S_)
                    _assert_rel(got[b:b + 1], want, 1e-5, f"dice loss sample {b}")
            self.check("f1_dice_loss", chk_loss)
        if self.measure("f1_dice_grad", 4 * (2 * n + 3 * B),
                        lambda: L.run("dice_loss_grad", [p, t, sums], [dx], ((n + 255) // 256, 1, 1), [B, S_]), 1):
            def chk_grad():
                sm = L.read(sums, 0, 3 * B)
                for b in ends:
                    want = _oracle_shaders().dice_loss_grad(L.read(p, b * S_, S_), L.read(t, b * S_, S_),
                                                            sm[3 * b:3 * b + 3], 1, S_, divisor=B)
                    _assert_bits(L.read(dx, b * S_, S_), want, f"dice grad sample {b}")
            self.check("f1_dice_grad", chk_grad)
        for h in (p, t, sums, loss, dx):
            lib.ReleaseBuffer(h)

    def _layout(self):
        """The layout ops beside the path at UNet-like sizes (every tensor larger than
        L2 or close to it), dispatched by reference shader name with the reference's
        cbuffer words: nearest 2x upsample and its gradient, channel concat of two
        tensors and one slice back, 2x2 max pooling (the shader alone, and
        MaxPoolForwardFused + MaxPoolBackwardFused as MaxPool2D runs them), and
        the conv output / gradient reshapes with ReLU.  No reference config sizes
        these ops; the shapes are synthetic.  Checks cover the first and last
        sample of each output (sample 0 of the conv reshapes)."""
        L, C, lib = self.L, self.C, self.lib
        for name in ("upsample", "upsample_backward", "concat_insert", "slice", "maxpool_forward", "conv_reshape",
                     "conv_grad_reshape_relu"):
            lib.CompileShader(name.encode(), "")
        B, Ch, H, W = 32, 128, 64, 64
        n_in, n_up = B * Ch * H * W, B * Ch * 4 * H * W              # 16.8M and 67M floats
        pin, pup = Ch * H * W, Ch * 4 * H * W                         # floats per sample
        seed = 5 + 1000 * self.rank
        x, y, dx, z, cat = L.new(n_in), L.new(n_up), L.new(n_in), L.new(n_up), L.new(2 * n_up)
        L.fill(x, seed, 20, 1, 0.0, 1.0)
        L.fill(z, seed, 21, 1, 0.0, 1.0)
        up = [B, Ch, H, W, 2 * H, 2 * W, 2, 2]
        ends = (0, B - 1)

        def per_sample(what, fn):
            def chk():
                for b in ends:
                    got, want = fn(b)
                    _assert_bits(got, want, f"{what} sample {b}")
            return chk
        if self.measure("f3_upsample2x_fwd", 4 * (n_in + n_up),
                        lambda: L.run("upsample", [x], [y], ((n_up + 255) // 256, 1, 1), up), 1):
            self.check("f3_upsample2x_fwd", per_sample("upsample", lambda b: (
                L.read(y, b * pup, pup),
                _oracle_shaders().upsample(L.read(x, b * pin, pin), 1, Ch, H, W, 2 * H, 2 * W, 2, 2))))
        if self.measure("f3_upsample2x_bwd", 4 * (n_in + n_up),
                        lambda: L.run("upsample_backward", [y], [dx], ((n_in + 255) // 256, 1, 1), up), 1):
            self.check("f3_upsample2x_bwd", per_sample("upsample_backward", lambda b: (
                L.read(dx, b * pin, pin),
                _oracle_shaders().upsample_backward(L.read(y, b * pup, pup), 1, Ch, H, W, 2 * H, 2 * W, 2, 2))))
        Sp = 4 * H * W
        grp = ((n_up + 255) // 256, 1, 1)

        def concat():
            L.run("concat_insert", [y], [cat], grp, [B, Ch, Sp, 2 * Ch, 0])
            L.run("concat_insert", [z], [cat], grp, [B, Ch, Sp, 2 * Ch, Ch])
        if self.measure("f3_concat", 4 * 4 * n_up, concat, 2):
            self.check("f3_concat", per_sample("concat", lambda b: (
                L.read(cat, b * 2 * pup, 2 * pup), np.concatenate([L.read(y, b * pup, pup), L.read(z, b * pup, pup)]))))
        zin = {b: L.read(cat, b * 2 * pup + pup, pup) for b in ends} if self.parity.enabled else {}
        if self.measure("f3_slice", 4 * 2 * n_up, lambda: L.run("slice", [cat], [z], grp, [B, Ch, Sp, 2 * Ch, Ch]), 1):
            self.check("f3_slice", per_sample("slice", lambda b: (L.read(z, b * pup, pup), zin[b])))
        po, pi = L.new(n_in), L.new(n_in)
        pool_groups = ((W + 15) // 16, (H + 15) // 16, B * Ch)
        if self.measure("f3_maxpool2x2_fwd", 4 * (n_up + 2 * n_in),
                        lambda: L.run("maxpool_forward", [y], [po, pi], pool_groups,
                                      [B, Ch, 2 * H, 2 * W, 2, 2, H, W]), 1):
            def chk():
                S = _oracle_shaders()
                for b in ends:
                    _, v, ix = S.maxpool_forward(L.read(y, b * pup, pup), 1, Ch, 2 * H, 2 * W, 2, 2, H, W)
                    _assert_bits(L.read(po, b * pin, pin), v, f"maxpool values sample {b}")
                    got = L.read(pi, b * pin, pin, np.uint32).astype(np.int64)
                    assert np.array_equal(got, ix.astype(np.int64) + b * pup), f"maxpool indices sample {b}"
            self.check("f3_maxpool2x2_fwd", chk)

        kept = []                                     # the last call's outputs, kept for the check

        def fused():                                  # MaxPool2D.forward + backward (nn_engine.py:1018-1047)
            pidx = C.c_void_p()
            o = lib.MaxPoolForwardFused(y, B, Ch, 2 * H, 2 * W, 2, 2, C.byref(pidx))
            d = lib.MaxPoolBackwardFused(po, pidx, B, Ch, H, W, n_up)     # releases the index buffer
            if not (o and d):
                raise RuntimeError("MaxPool*Fused: " + lib.dct_last_error().decode())
            for h in kept:
                lib.ReleaseBuffer(h)
            kept[:] = [o, d]
        if self.measure("f3_maxpool2x2_fused_fwd_bwd", 4 * (n_up + 2 * n_in) + 4 * (2 * n_in + n_up), fused, 3):
            def chk():
                S = _oracle_shaders()
                o, d = kept
                for b in ends:
                    _, v, ix = S.maxpool_forward(L.read(y, b * pup, pup), 1, Ch, 2 * H, 2 * W, 2, 2, H, W)
                    _assert_bits(L.read(o, b * pin, pin), v, f"MaxPoolForwardFused sample {b}")
                    want = S.maxpool_backward(np.zeros(pup, np.float32), L.read(po, b * pin, pin), ix, 1, Ch, H, W)
                    _assert_bits(L.read(d, b * pup, pup), want, f"MaxPoolBackwardFused sample {b}")
            self.check("f3_maxpool2x2_fused_fwd_bwd", chk)
        for h in kept + [x, dx, z, cat, po, pi]:
            lib.ReleaseBuffer(h)
        OC, Bc, P = 256, 64, 64 * 64
        nconv = OC * Bc * P                                           # 67M floats
        mm, bias, co, gr = L.new(nconv), L.new(OC), y, L.new(nconv)
        L.fill(mm, seed, 22, 1, 0.0, 1.0)
        L.fill(bias, seed, 23, 1, 0.0, 0.1)
        cgrp = ((Bc * P + 15) // 16, (OC + 15) // 16, 1)
        if self.measure("f4_conv_reshape_relu", 4 * (2 * nconv + OC),
                        lambda: L.run("conv_reshape", [mm, bias], [co], cgrp, [Bc, OC, 64, 64, 1]), 1):
            def chk():
                dst, val = _oracle_shaders().conv_reshape(L.read(mm, 0, nconv), L.read(bias, 0, OC), Bc, OC, 64, 64, 1,
                                                          lim_bp=P)                      # sample 0
                _assert_bits(L.read(co, 0, OC * P)[dst], val, "conv_reshape sample 0")
            self.check("f4_conv_reshape_relu", chk)
        if self.measure("f4_conv_grad_reshape_relu", 4 * 3 * nconv,
                        lambda: L.run("conv_grad_reshape_relu", [mm, co], [gr], cgrp,
                                      [Bc, 0, 0, 0, OC, 0, 0, 64, 64]), 1):
            def chk():
                dst, val = _oracle_shaders().conv_grad_reshape(L.read(mm, 0, OC * P), 1, OC, 64, 64,
                                                               fwd=L.read(co, 0, OC * P))
                # sample 0 of the gradient sits at [oc][0 .. P) of each [OC][Bc*P] row
                oc, pix = dst // P, dst % P
                _assert_bits(L.read(gr, 0, nconv)[oc * (Bc * P) + pix], val, "conv_grad_reshape_relu sample 0")
            self.check("f4_conv_grad_reshape_relu", chk)
        for h in (mm, bias, y, gr):
            lib.ReleaseBuffer(h)


class _OneRank:
    def __init__(self, rank=0):
        self.rank, self.world = rank, 1

    def gather(self, a):
        return [np.asarray(a, np.float64)]

    def all_true(self, flags):
        return list(flags)


def per_op_suite(L: "Lib", rank: int, iters: int = 10, only: str | None = None, warmup: int = 3, comm=None,
                 ranks=None, split: str = "weak", parity: Parity | None = None, sections=None):
    """Per-op timings (name -> gbs, ms, bytes, launches) of one Suite pass."""
    return Suite(L, ranks if ranks is not None else _OneRank(rank), comm, split, parity, iters, warmup,
                 only).run(sections)


# ---------------------------------------------------------------------------
# CPU baseline: the NumPy restatement (oracle) on this host's cores
# ---------------------------------------------------------------------------
def cpu_c2_sample(threads: int, rows: int = 1024, reps: int = 3, min_seconds: float = 0.0, warmup: int = 1):
    """Time the 11 C2 ops in NumPy (oracle semantics) on a `rows`-row sample of A.

    Returns (GB/s over algorithmic bytes, seconds per pass, description, timed passes)."""
    from oracle.threaded import c2_sample
    return c2_sample(threads, rows=rows, reps=reps, min_seconds=min_seconds, warmup=warmup)


def cpu_other_configs(threads: int) -> dict:
    """The oracle's arithmetic for C1 (whole, one thread), C3, C4, C5a and C5b (bounded
    samples on `threads` threads), about 1-2 s each."""
    from oracle import threaded as T
    out = {}
    for key, fn in (("c1", T.c1_sample), ("c3", T.c3_sample), ("c4", T.c4_sample), ("c5a", T.c5a_sample),
                    ("c5b", T.c5b_sample)):
        gbs, secs, desc = fn(threads)
        out[key] = {"gbs": round(gbs, 2), "s_per_pass": round(secs, 6 if key == "c1" else 4), "sample": desc}
        if key == "c1":
            out[key]["us_per_step"] = round(secs * 1e6, 1)
    return out


def c2_config(world: int) -> dict:
    """The workload both arms report."""
    step_bytes = len(C2_BINARY) * ROWBCAST_BYTES + len(C2_OUTER) * OUTER_BYTES + len(C2_UNARY) * UNARY_BYTES
    return {"workload": "C2: A[8192,8192] op B[1,8192] (add/sub/mul/div/maximum), "
                        "C[64,1,4096] op D[1,512,4096] (mul/add), exp/log(|x|+1)/tanh/sigmoid on A",
            "per_rank_rows": A_ROWS, "global_rows": A_ROWS * world,
            "parallelism": f"dp{world} (rows sharded, no collective)",
            "l2": "inputs larger than L2 (A = 256 MB; outputs 256-512 MB written fresh)",
            "step_bytes": step_bytes}


def reference_arm(args, rank: int):
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    # one step = one pass of the bounded C2 sample (1/8 of the rows); W + K passes
    gbs, secs, sample, passes = cpu_c2_sample(threads, reps=max(1, args.steps), warmup=max(0, args.warmup))
    line = {
        "metric": METRIC, "impl": "reference", "value": round(gbs, 2), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": passes, "warmup": args.warmup, "ms_per_step": round(secs * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": c2_config(args.gpus),
        "cpu_baseline": {"value": round(gbs, 2), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


_SHORT = {"c1_dense_step_eager": "c1.eager", "c1_dense_step_graph": "c1.graph", "c3_fullsum_2^30": "c3.full",
          "c4_softmax_ce_fused": "c4", "c5a_adam_1.5e9": "c5a", "c5b_batchnorm_fwd": "c5b.f",
          "c5b_batchnorm_bwd": "c5b.b", "f3_upsample2x_fwd": "f3.up", "f3_upsample2x_bwd": "f3.upb",
          "f3_concat": "f3.cat", "f3_slice": "f3.slice", "f3_maxpool2x2_fwd": "f3.pool",
          "f3_maxpool2x2_fused_fwd_bwd": "f3.poolfb", "f4_conv_reshape_relu": "f4.conv",
          "f4_conv_grad_reshape_relu": "f4.convg", "f1_dice_sums": "f1.sums", "f1_dice_loss": "f1.loss",
          "f1_dice_grad": "f1.grad"}


def short(name: str) -> str:
    """Short op key for the compact maps at the end of the line."""
    if name in _SHORT:
        return _SHORT[name]
    if name.startswith("c3_") and "_axis" in name:
        op, ax = name[3:].split("_axis")
        return f"c3.{op}{'1' if ax == '-1' else '0'}"
    for pre, rep in (("c2_rowbcast_", "c2."), ("c2_outer_", "c2.o"), ("c2_unary_", "c2.")):
        if name.startswith(pre):
            return rep + name[len(pre):]
    return name


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="dct", choices=("dct", "reference"))
    ap.add_argument("--no-per-op", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-verify", action="store_true", help="skip reading back and checking the timed outputs")
    ap.add_argument("--no-strong", action="store_true", help="at N > 1, skip the fixed-global-size pass")
    ap.add_argument("--only", default=None, help="profiling mode: run one op (a C2 op such as c2_rowbcast_add, "
                    "or a per_op name; c3_fullsum_2^28_small and c5a_adam_1.5e8_small are smaller cases of "
                    "the same kernels for profiler captures) --warmup + --steps times and print its timing only")
    args = ap.parse_args()
    if args.impl == "reference":
        # the CPU arm needs no GPU and no process group: rank 0 alone runs it,
        # the other ranks of a torchrun launch exit 0 at once
        return reference_arm(args, int(os.environ.get("RANK", "0")))
    ranks = Ranks(args.gpus)
    os.environ.setdefault("DCT_DEVICE", str(ranks.local))
    L = Lib()
    if args.only and not args.only.startswith("c2_"):
        res = per_op_suite(L, ranks.rank, iters=args.steps, only=args.only, warmup=args.warmup)
        print(json.dumps({"only": args.only, **res.get(args.only, {})}))
        ranks.close()
        return 0
    c2 = C2(L, ranks.rank, only=args.only)
    lib = L.lib
    if args.only:
        name, nbytes, fn = c2.ops[0]
        for _ in range(args.warmup):
            fn()
        ms = L.time(fn, args.steps) / max(1, args.steps)
        print(json.dumps({"only": name, "ms": round(ms, 4), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                          "launches": args.warmup + args.steps}))
        ranks.close()
        return 0
    parity = Parity(not args.no_verify)
    parity_strong = Parity(not args.no_verify)
    # per-op timing of the step's kernels (dominant kernel + roofline)
    ops = {}
    for name, nbytes, fn in c2.ops:
        for _ in range(2):
            fn()
        ms = L.time(fn, 5) / 5
        ops[name] = {"ms": ms, "bytes": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9}
    for _ in range(max(3, args.warmup)):
        c2.step()
    lib.dct_synchronize()
    L.launches = 0
    ranks.barrier()
    lib.dct_synchronize()
    bus = L.C.create_string_buffer(64)
    lib.dct_pci_bus_id(bus, 64)
    with Clocks(bus.value.decode()) as clk:
        ms = L.time(c2.step, args.steps)
        lib.dct_synchronize()
    ranks.barrier()
    launches = L.launches
    ms_max = ranks.max(ms)
    world = ranks.world
    total_bytes = c2.step_bytes * args.steps * world
    value = total_bytes / (ms_max * 1e-3) / 1e9
    peak, peak_kind = _peaks()
    verify_c2(L, c2, parity)
    # dominant kernel family: the one with the largest share of the step time
    fams = {}
    for name in ops:
        fams.setdefault("_".join(name.split("_")[:2]), []).append(name)
    dom_f = max(fams, key=lambda f: sum(ops[n]["ms"] for n in fams[f]))
    dom_ms = sum(ops[n]["ms"] for n in fams[dom_f]) / len(fams[dom_f])
    dom_bytes = ops[fams[dom_f][0]]["bytes"]
    dom_share = sum(ops[n]["ms"] for n in fams[dom_f]) / sum(v["ms"] for v in ops.values())
    dom = f"{dom_f} x{len(fams[dom_f])} ({', '.join(n.split('_', 2)[2] for n in fams[dom_f])})"
    achieved = dom_bytes / (dom_ms * 1e-3) / 1e9
    traffic = NCU_TRAFFIC_BYTES.get(dom_f)
    e2e = None
    if not args.no_e2e:
        dt, h2d, d2h = run_e2e(L, c2, steps=max(1, min(args.steps, 3)), warmup=1)
        nst = max(1, min(args.steps, 3))
        e2e_val = ranks.sum(c2.step_bytes * nst) / ranks.max(dt) / 1e9
        e2e = {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
        # the step's host copies at the measured pinned-copy rates: the floor for e2e
        lh2d, ld2h = link_bandwidth(L)
        floor_s = h2d / (lh2d * 1e9) + d2h / (ld2h * 1e9)
        step_s = ranks.max(dt) / nst
        e2e["link"] = {"h2d_gbs": round(lh2d, 1), "d2h_gbs": round(ld2h, 1),
                       "copy_floor_ms_per_step": round(floor_s * 1e3, 2),
                       "ms_per_step": round(step_s * 1e3, 2), "frac_of_copy_floor": round(floor_s / step_s, 3)}
        if world > 1:                      # every rank copies its own batch over a shared host
            e2e["per_rank_gbs"] = round(e2e_val / world, 2)
    per_op, strong = {}, {}
    exchange = None
    clk_ops = None
    if not args.no_per_op:
        comm = None
        if world > 1:
            from directcompute_torch_b200.dist import Communicator
            comm = Communicator.from_process_group(timeout_s=120)
            exchange = "peer memory (NVLink, CUDA IPC)" if comm.peer_exchange else "NCCL all-gather"
        with Clocks(bus.value.decode(), period_s=0.02) as clk2:
            per_op = per_op_suite(L, ranks.rank, comm=comm, ranks=ranks, parity=parity)
            if world > 1 and not args.no_strong:
                strong = per_op_suite(L, ranks.rank, comm=comm, ranks=ranks, split="strong",
                                      parity=parity_strong, sections=STRONG_SECTIONS)
        clk_ops = clk2.summary()
        if comm is not None:
            comm.close()
        if world > 1:
            for res in (per_op, strong):
                for k in res:
                    res[k]["ms"] = ranks.max(res[k]["ms"])
                    res[k]["gbs"] = round(res[k]["bytes"] * world / (res[k]["ms"] * 1e-3) / 1e9, 1)
    for k, v in ops.items():
        ms_k = ranks.max(v["ms"]) if world > 1 else v["ms"]     # every rank ran its shard: whole-job rate
        per_op[k] = {"gbs": round(v["bytes"] * world / (ms_k * 1e-3) / 1e9, 1), "ms": round(ms_k, 4),
                     "bytes": v["bytes"], "launches": 1}
    for res in (per_op, strong):
        for v in res.values():
            v["frac_of_measured_hbm"] = round(v["gbs"] / (peak * world), 3)
            v["frac_of_8TBs"] = round(v["gbs"] / (NOMINAL_HBM_GBS * world), 3)
    cpu = None
    if ranks.rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        gbs, secs, sample, _ = cpu_c2_sample(threads, reps=3, min_seconds=6.0)      # about 6 s of CPU work
        cpu = {"value": round(gbs, 2), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample,
               "other_configs": cpu_other_configs(threads)}
    par = parity.finish(ranks)
    par_strong = parity_strong.finish(ranks)
    clocks = clk.summary()
    err = lib.dct_error_code()
    if err:
        raise RuntimeError("libdct_cuda reported: " + lib.dct_last_error().decode())
    if ranks.rank == 0:
        if strong:
            strong_c = {short(k): [v["ms"], v["frac_of_measured_hbm"]] for k, v in strong.items()}
        elif world == 1 and per_op:          # at N = 1 the split configs are the single-GPU ones
            strong_c = {short(k): [per_op[k]["ms"], per_op[k]["frac_of_measured_hbm"]]
                        for k in ("c3_sum_axis0", "c3_argmax_axis0", "c3_fullsum_2^30", "c4_softmax_ce_fused",
                                  "c5a_adam_1.5e9", "c5b_batchnorm_fwd", "c5b_batchnorm_bwd") if k in per_op}
        else:
            strong_c = {}
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (on-device Philox4x32-10)",
            "config": c2_config(world),
            "frac_of_measured_hbm": round(value / (peak * world), 3),
            "frac_of_8TBs": round(value / (NOMINAL_HBM_GBS * world), 3),
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, burst)", "unit": "GB/s",
                         "frac": round(achieved / peak, 3), "traffic": traffic, "share_of_step": round(dom_share, 3),
                         "algorithmic_bytes_per_launch": dom_bytes},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clocks,
            "clocks_per_op": clk_ops,
            "sharded_exchange": exchange,
            "per_op": per_op,
            "strong_detail": strong or None,
            "parity_notes": {**parity.msg, **{"strong " + k: v for k, v in parity_strong.msg.items()}} or None,
            "parity": {short(k): v for k, v in par.items()},
            # the compact tail (the driver keeps the line's last 1500 characters)
            "c1_us": {k.split("_")[-1]: per_op[k].get("us_per_step")
                      for k in ("c1_dense_step_eager", "c1_dense_step_graph") if k in per_op},
            "per_op_frac": {short(k): round(v["frac_of_measured_hbm"], 3) for k, v in per_op.items()
                            if not k.startswith("c1_")},
            "strong": strong_c,
            "parity_failed": sorted([short(k) for k, v in par.items() if not v] +
                                    ["strong " + short(k) for k, v in par_strong.items() if not v]),
            "parity_all": (all(par.values()) if par else None),
            "parity_strong_all": (all(par_strong.values()) if par_strong else None),
        }
        print(json.dumps(line, separators=(",", ":")))
    ranks.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
