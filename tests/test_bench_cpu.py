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
