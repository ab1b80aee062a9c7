"""bench.py's reference arm on the host: one JSON line from rank 0 with the contract's keys, and
nothing (exit 0) from any other rank. It runs the oracle port on the CPU, so no GPU is needed, and
it must not load this repository's CUDA library (the arm times the reference alone)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CMD = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "cpu_plumbing",
       "--steps", "2", "--warmup", "3"]


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run(CMD, cwd=ROOT, capture_output=True, text=True, timeout=300, env=env, check=True).stdout


def test_reference_arm_line():
    out = _run({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0"})
    lines = [x for x in out.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["unit"] == "TFLOP/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["ms_per_step"] > 0 and line["steps"] >= 1
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == line["value"] and cpu["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["gpu_launches"] == 0
    assert line["config"]["workload"] == "cpu_plumbing"
    assert line["repo_libraries_mapped"] == []
    assert line["scaling"] == "strong" and line["config"]["layers_per_job"] == 1


def test_both_arms_report_the_same_config():
    import argparse
    import importlib.util
    spec = importlib.util.spec_from_file_location("_bench_under_test", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    w = bench.WORKLOADS["dit14b"]
    for scaling in ("strong", "weak"):
        for n in (1, 8):
            args = argparse.Namespace(steps=20, warmup=5, scaling=scaling, graph=False)
            ours = bench.base_line(args, w, n, 17.0, 700.0)
            ref = bench.base_line(args, w, n, 2e4, 0.6, impl="reference")
            assert ours["config"] == ref["config"]
            assert ours["config"]["layers_per_job"] == (1 if scaling == "strong" else n)


def test_reference_arm_other_ranks_print_nothing():
    out = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert not [x for x in out.splitlines() if x.startswith("{")]


def test_clock_sampler_keeps_the_timed_window():
    # A stand-in for NVML: the SM clock drops and the power-cap reason comes on after the first
    # samples. The summary keeps only samples inside the window the timed region reports.
    import importlib.util
    import time
    import types
    spec = importlib.util.spec_from_file_location("_bench_clock_test", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    calls = {"n": 0}

    def clock(h, kind):
        calls["n"] += 1
        return 1965 if calls["n"] <= 3 else 1700

    start = time.monotonic()

    def fields(h, ids):  # cumulative power-cap timer: capped half of the time, the other reasons never
        ns = int((time.monotonic() - start) * 0.5e9)
        return [types.SimpleNamespace(nvmlReturn=0, value=types.SimpleNamespace(ullVal=ns if i == 11 else 0))
                for i in ids]

    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=1, nvmlInit=lambda: None, nvmlShutdown=lambda: None, nvmlDeviceGetFieldValues=fields,
        NVML_FI_DEV_CLOCKS_EVENT_REASON_SW_POWER_CAP=11, NVML_FI_DEV_CLOCKS_EVENT_REASON_HW_POWER_BRAKE_SLOWDOWN=12,
        NVML_FI_DEV_CLOCKS_EVENT_REASON_HW_THERM_SLOWDOWN=13, NVML_FI_DEV_CLOCKS_EVENT_REASON_SW_THERM_SLOWDOWN=14,
        nvmlDeviceGetHandleByUUID=lambda u: "h", nvmlDeviceGetHandleByIndex=lambda i: "h",
        nvmlDeviceGetMaxClockInfo=lambda h, kind: 1965, nvmlDeviceGetClockInfo=clock,
        nvmlDeviceGetCurrentClocksEventReasons=lambda h: 0x4 if calls["n"] > 3 else 0x1,
        nvmlDeviceGetPowerUsage=lambda h: 990000)
    with bench.ClockSampler("cpu", nvml=fake) as clk:
        time.sleep(0.1)
        clk.begin()
        time.sleep(0.1)
        clk.end()
    s = clk.summary()
    assert s["sm_mhz"] == 1700 and s["sm_max_mhz"] == 1965 and s["samples"] >= 5
    assert s["reasons"] == ["sw_power_cap"] and s["power_w_max"] == 990.0
    assert "timed region" in s["source"]
    # the timers' span starts at the last snapshot before the region and ends past it: it covers
    # the region and NVML's refresh period after it
    trail = bench.ClockSampler.TRAIL_S * 1e3
    assert 90 <= s["region_ms"] and s["region_ms"] + trail <= s["throttle_span_ms"] <= s["region_ms"] + trail + 60
    t = s["throttle_ms"]
    assert 0.45 * s["throttle_span_ms"] <= t["sw_power_cap"] <= 0.55 * s["throttle_span_ms"]
    assert t["hw_power_brake_slowdown"] == t["hw_thermal_slowdown"] == t["sw_thermal_slowdown"] == 0
