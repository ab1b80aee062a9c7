"""bench.py's reference arm on the host: one JSON line from rank 0 with the contract's keys, and
nothing (exit 0) from any other rank. It runs the oracle port on the CPU, so no GPU is needed."""
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


def test_reference_arm_other_ranks_print_nothing():
    out = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert not [x for x in out.splitlines() if x.startswith("{")]
