"""bench.py host logic on CPU: metric names, clock-sample windowing, the
roofline traffic lookup, and the JSON line of the reference arm."""
from __future__ import annotations

import importlib.util
import json
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_metric_names_are_shared_by_both_arms(bench):
    assert bench.metric_name("cfg4", "GB/s") == bench.METRIC
    assert bench.metric_name("cfg3", "GB/s") == bench.METRIC
    assert bench.metric_name("cfg5-t512", "TFLOP/s") == "cfg5-t512 chunked prefill attention TFLOP/s"
    assert bench.metric_name("scatter", "GB/s") == "scatter KV scatter GB/s"
    assert bench.metric_name("qkv-decode", "GB/s") == "qkv-decode fused QKV projection + KV write GB/s"


def test_clock_summary_keeps_only_the_timed_window(bench):
    pynvml = pytest.importorskip("pynvml")
    c = bench.ClockSampler([0], period_s=0.002)
    cap = pynvml.nvmlClocksEventReasonSwPowerCap
    c.samples = [(0.0, 1000.0, 1965.0, 0), (1.0, 1965.0, 1965.0, 0), (1.5, 1900.0, 1965.0, cap),
                 (3.0, 800.0, 1965.0, 0)]
    c._t0, c._t1 = 0.9, 2.0
    s = c.summary()
    assert s["samples"] == 2 and s["sm_mhz"] == pytest.approx(1932.5)
    assert s["reasons"] == ["sw_power_cap"] and "window" not in s


def test_clock_summary_widens_a_window_shorter_than_the_period(bench):
    pytest.importorskip("pynvml")
    c = bench.ClockSampler([0], period_s=0.002)
    c.samples = [(1.000, 1965.0, 1965.0, 0), (1.0025, 1965.0, 1965.0, 0), (5.0, 500.0, 1965.0, 0)]
    c._t0, c._t1 = 1.0005, 1.0015  # no sample inside
    s = c.summary()
    assert s["samples"] == 2 and s["sm_mhz"] == 1965.0 and "window" in s
    c.samples = []
    assert c.summary()["samples"] == 0


def test_roofline_traffic_comes_from_committed_profiles(bench):
    for wl in ("cfg4", "cfg3", "qkv-prefill", "qkv-decode"):
        t = bench.traffic_from_profile(wl, 1e9)
        assert t is not None and t > 0, wl
    # configuration 3's summary is a DRAM/algorithmic ratio, applied per launch
    assert bench.traffic_from_profile("cfg3", 2e9) == pytest.approx(
        2 * bench.traffic_from_profile("cfg3", 1e9))
    assert bench.traffic_from_profile("scatter", 1e9) is None
    assert bench.traffic_from_profile(None, 1e9) is None


def test_default_run_names_every_extra_workload(bench):
    assert set(bench.EXTRA_WORKLOADS) == {"cfg3", "cfg3-f32", "cfg5-t512", "cfg5-t64", "scatter",
                                          "qkv-prefill", "qkv-decode"}


def test_usable_cpus_is_positive(bench):
    assert bench.usable_cpus() >= 1


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference",
                          "--workload", "scatter", "--steps", "1", "--warmup", "3"],
                         capture_output=True, text=True, timeout=600, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["value"] > 0
    assert d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 3
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"]


def test_warmup_below_three_is_rejected():
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference",
                          "--workload", "scatter", "--steps", "1", "--warmup", "2"],
                         capture_output=True, text=True, timeout=120, cwd=REPO)
    assert out.returncode != 0 and "warmup" in out.stderr


def test_cpu_baseline_sample_with_one_thread(bench):
    r = bench.cpu_reference_sample("scatter", steps=1, warmup=0, threads=1)
    assert r["cores"] == 1 and r["value"] > 0 and r["kind"] == "port"
    assert isinstance(bench.cpu_model(), str) and bench.cpu_model()
