"""bench.py's reference arm on CPU: the JSON line the driver reads (no GPU needed).

`bench.py --impl reference` times the reference's CPU arithmetic for the C2
workload (the NumPy restatement, as the reference's own CPU path is NumPy).
Launched alone or by torchrun, rank 0 prints exactly one line with the
contract's keys and every rank exits 0.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = {"metric", "impl", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _lines(out: str):
    return [json.loads(s) for s in out.splitlines() if s.startswith("{")]


def _check(line, n_gpus):
    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and line["n_gpus"] == n_gpus and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert "workload" in line["config"]


def test_reference_arm_single_process():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1
    _check(lines[0], 1)


def test_reference_arm_under_torchrun_prints_once():
    pytest.importorskip("torch")
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", "29637", "bench.py", "--impl", "reference",
                        "--gpus", "2", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _lines(r.stdout)
    assert len(lines) == 1
    _check(lines[0], 2)


def test_clock_record_with_a_fake_nvml(monkeypatch):
    """bench.Clocks samples NVML during the timed region: median / minimum SM clock,
    the active clock-event reasons by name, the sample count and the measured period."""
    import time
    import types
    state = {"k": 0}
    N = types.ModuleType("pynvml")
    N.NVML_CLOCK_SM = 1
    N.nvmlInit = lambda: None
    N.nvmlDeviceGetHandleByPciBusId = lambda bus: 0
    N.nvmlDeviceGetMaxClockInfo = lambda h, c: 1965

    def clock(h, c):
        state["k"] += 1
        return 1965 if state["k"] % 3 else 1732
    N.nvmlDeviceGetClockInfo = clock
    N.nvmlDeviceGetPowerUsage = lambda h: 650000                   # mW
    N.nvmlDeviceGetCurrentClocksEventReasons = lambda h: 0x4 | 0x40  # power cap + HW thermal
    monkeypatch.setitem(sys.modules, "pynvml", N)
    sys.path.insert(0, ROOT)
    try:
        import bench
    finally:
        sys.path.remove(ROOT)
    with bench.Clocks("0000:00:00.0", period_s=0.002) as clk:
        time.sleep(0.1)
    rec = clk.summary()
    assert rec["samples"] >= 10 and rec["sm_max_mhz"] == 1965
    assert rec["sm_mhz"] == 1965.0 and rec["sm_min_mhz"] == 1732.0
    assert rec["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]
    assert rec["power_w_max"] == 650.0 and 1.5 < rec["period_ms"] < 20
    # no NVML at all: the record says so instead of inventing clocks
    monkeypatch.setitem(sys.modules, "pynvml", types.ModuleType("pynvml"))
    with bench.Clocks("0000:00:00.0") as clk:
        pass
    rec = clk.summary()
    assert rec["samples"] == 0 and rec["reasons"] == ["unsampled"] and rec["sm_mhz"] is None


def test_compact_maps_and_parity_bookkeeping():
    """The short op keys the line ends with are unique, and a failed check is recorded
    (with its message) without stopping the others."""
    sys.path.insert(0, ROOT)
    import bench
    names = [n for sec in bench.PER_OP_SECTIONS.values() for n in sec if "small" not in n]
    names += [f"c2_rowbcast_{o}" for o in bench.C2_BINARY] + [f"c2_outer_{o}" for o in bench.C2_OUTER]
    names += [f"c2_unary_{o}" for o in bench.C2_UNARY]
    keys = [bench.short(n) for n in names]
    assert len(set(keys)) == len(keys), keys
    p = bench.Parity(True)
    p.run("a", lambda: None)

    def bad():
        raise AssertionError("off by one ulp")
    p.run("b", bad)
    p.run("c", lambda: None)
    assert p.finish(bench._OneRank()) == {"a": True, "b": False, "c": True}
    assert "off by one" in p.msg["b"]
    q = bench.Parity(False)
    q.run("a", bad)
    assert q.finish(bench._OneRank()) == {}


def test_cpu_c1_sample_matches_the_oracle_and_times_a_step():
    """The C1 CPU baseline checks its vectorised NumPy chain against the oracle's
    formulas (it asserts bit equality before timing) and reports seconds per step."""
    from oracle import threaded as T
    gbs, secs, desc = T.c1_sample(1, reps=3, min_seconds=0.0)
    assert gbs > 0 and 0 < secs < 1.0
    assert "C1 whole" in desc and "1 thread" in desc
