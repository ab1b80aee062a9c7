#!/usr/bin/env python
"""Benchmark of the VMonarch attention hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|triton]
                    [--workload dit14b] [--scaling weak|strong] [--graph]

A step is one forward + backward of VMonarch attention over one synthetic layer of the workload
(default: the video-DiT 14B-class layer B=1, H=40, m=21, b=1560, D=128, 2 iterations, 1560 recomputed
tokens: the N~32K, H=40, D=128 configuration the metric is quoted on). The metric is effective
algorithmic TFLOP/s of forward+backward (FLOPs counted on unpadded shapes, 2 per multiply-add).

impl ours       this repository's CUDA path; `value` from inputs resident in HBM (every input and
                activation is > 126 MB, larger than L2, so no flush is needed), `e2e` through the public
                API with the step's inputs copied from pinned host memory and the loss read back.
impl reference  the reference's CPU path (the fp32 oracle restating the reference's PyTorch code)
                on the host cores, on a bounded sample (whole heads) of the same workload.
impl triton     the reference's own Triton kernels (installed in baseline/_ref) on the same GPU;
                reported for comparison, not part of the driver's contract.
Multi-GPU (torchrun): (batch x head) units are sharded with no collective on the hot path.
`--scaling strong` (default) splits one layer's heads over the ranks (rank g of N runs heads
[g*H/N, (g+1)*H/N)); after the timed region the outputs and gradients of every head are gathered
over NCCL and rank 0 checks two of them against its own single-GPU run. `--scaling weak` gives
every rank one full layer.
At N = 1 the line also carries the FlashEntropyAttention forward on the fea32k configuration
(B=1, H=24, N=32768, D=128), timed with CUDA events beside the reference's Triton forward when
baseline/_ref holds the reference.
"""
from __future__ import annotations

import argparse
import contextlib
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))



def _standalone(name: str, rel: str):
    """Loads one self-contained module of the package by path, without the package __init__ (which
    loads the CUDA library): the reference arm must not map this repository's library."""
    spec = importlib.util.spec_from_file_location(name, ROOT / rel)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


shard = _standalone("_vmb_bench_shard", "vmonarch_b200/shard.py")
_configs = _standalone("_vmb_bench_configs", "vmonarch_b200/configs.py")
WORKLOADS, Workload, make_inputs = _configs.WORKLOADS, _configs.Workload, _configs.make_inputs

METRIC = "VMonarch fwd+bwd effective TFLOP/s (N~32K, H=40, D=128, bf16)"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "triton"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="dit14b")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="strong")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--heads", type=int, default=0, help="run only this many heads of the layer (profiling)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--graph", action="store_true",
                    help="time `value` as replays of one CUDA graph holding the whole step (launch-bound sizes)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-verify", action="store_true", help="skip the gather + single-GPU check after timing")
    ap.add_argument("--no-fea-forward", action="store_true", help="skip the fea32k forward timing (N = 1)")
    ap.add_argument("--fwd-only", action="store_true", help="impl triton: time the forward alone")
    ap.add_argument("--fp8-r-step", action="store_true",
                    help="VMonarch R steps on e4m3 operands (opt-in extension; the default line is bf16)")
    ap.add_argument("--cpu-budget-s", type=float, default=150.0, help="wall-clock cap of the CPU reference arm")
    return ap.parse_args()


# ----------------------------------------------------------------------------------------- clocks
class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons of this GPU while the timed region runs.

    A host thread reads them through NVML (the library nvidia-smi reports from) continuously (a
    pass every 5-10 ms, a timer read included), each sample stamped with the host time; `begin()` / `end()` (called by `time_steps` at the
    synchronisations that bracket the timed region) restrict the summary to that span and
    snapshot NVML's cumulative per-reason throttle timers, so `throttle_ms` is the time the GPU
    spent in each reason over the timed region. The sampling thread snapshots the timers
    continuously (an NVML field read can take tens of ms, which must not delay the timed launches,
    nor leave the GPU idle before them); the begin reference is the last snapshot completed before
    the region started, so the timed span (`throttle_span_ms`, up to one read longer than the
    region, into the warm-up) covers the whole region and may over-count, never under-count; the
    end snapshot is read after the region's final synchronisation.
    NVML refreshes its readings (clocks, power, reasons and these timers) only every ~100 ms, so
    `end()` keeps the record open TRAIL_S past the region (the GPU is idle then; the timed region
    is over): every state NVML held during the region is seen, and a reason that starts just after
    it is counted too (the record may over-count, never under-count). Without NVML it falls back
    to `nvidia-smi -lms 200` over the whole `with` block. Reading clocks changes no GPU setting."""

    PERIOD_S = 0.005
    TRAIL_S = 0.12
    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    REASON_BITS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
                   "sw_power_cap": 0x4}

    def __init__(self, device: torch.device, nvml=None):
        self.uuid = None
        try:
            self.uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            pass
        self.nvml = nvml  # a stand-in module for tests; None: pynvml if importable
        self.handle = None
        self.samples = []  # (host time, sm MHz, reason bits, power W)
        self.max_mhz = None
        self.span = None
        self.t0 = None
        self.snaps = []  # (host time the read started, host time it returned, timers)
        self.throttle_ms = None
        self.throttle_span_ms = None
        self.region_ms = None
        self.stop = None
        self.thread = None
        self.proc = None
        self.tmp = None

    def window(self, t0: float, t1: float) -> None:
        self.span = (t0, t1)

    # NVML field ids of the cumulative throttle timers (ns), by reason
    def _timer_fields(self):
        nv = self.nvml
        names = (("sw_power_cap", "NVML_FI_DEV_CLOCKS_EVENT_REASON_SW_POWER_CAP"),
                 ("hw_power_brake_slowdown", "NVML_FI_DEV_CLOCKS_EVENT_REASON_HW_POWER_BRAKE_SLOWDOWN"),
                 ("hw_thermal_slowdown", "NVML_FI_DEV_CLOCKS_EVENT_REASON_HW_THERM_SLOWDOWN"),
                 ("sw_thermal_slowdown", "NVML_FI_DEV_CLOCKS_EVENT_REASON_SW_THERM_SLOWDOWN"))
        return [(n, getattr(nv, f)) for n, f in names if hasattr(nv, f)]

    def _timers(self):
        if self.handle is None or not hasattr(self.nvml, "nvmlDeviceGetFieldValues"):
            return None
        try:
            fields = self._timer_fields()
            vals = self.nvml.nvmlDeviceGetFieldValues(self.handle, [f for _, f in fields])
            return {n: v.value.ullVal for (n, _), v in zip(fields, vals) if v.nvmlReturn == 0}
        except Exception:
            return None

    def begin(self) -> None:
        self.t0 = time.monotonic()

    def end(self) -> None:
        t1 = time.monotonic()
        if self.thread is not None:
            time.sleep(self.TRAIL_S)  # past NVML's refresh period: the region's state is published
        timers1 = self._timers()
        if self.t0 is None:
            return
        self.region_ms = round((t1 - self.t0) * 1e3, 2)
        t1 = time.monotonic()
        self.window(self.t0, t1)
        before = [sn for sn in list(self.snaps) if sn[1] <= self.t0 and sn[2]]
        if before and timers1 is not None:
            ts, _, timers0 = before[-1]
            self.throttle_ms = {n: round((timers1[n] - timers0[n]) / 1e6, 2) for n in timers1 if n in timers0}
            self.throttle_span_ms = round((t1 - ts) * 1e3, 2)

    def _open_nvml(self) -> bool:
        try:
            if self.nvml is None:
                import pynvml
                self.nvml = pynvml
            nv = self.nvml
            nv.nvmlInit()
            if self.uuid:
                self.handle = nv.nvmlDeviceGetHandleByUUID(self.uuid)
            else:  # no CUDA device properties: the first GPU (NVML numbering)
                self.handle = nv.nvmlDeviceGetHandleByIndex(0)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.handle, nv.NVML_CLOCK_SM))
            return True
        except Exception:
            self.handle = None
            return False

    def _poll(self) -> None:
        nv, h = self.nvml, self.handle
        reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop.is_set():
            ts = time.monotonic()
            timers = self._timers()
            if timers:
                self.snaps.append((ts, time.monotonic(), timers))
            try:
                self.samples.append((time.monotonic(), float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                     int(reasons(h)), nv.nvmlDeviceGetPowerUsage(h) / 1000.0))
            except Exception:
                pass
            self.stop.wait(self.PERIOD_S)

    def __enter__(self):
        if self._open_nvml():
            # one snapshot before the warm-up (the GPU is idle here), so a region whose warm-up is
            # shorter than an NVML read still has a reference taken before it
            t = time.monotonic()
            timers = self._timers()
            if timers:
                self.snaps.append((t, time.monotonic(), timers))
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return self
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.thread is not None:
            rows = self.samples
            if self.span is not None:
                inside = [r for r in rows if self.span[0] <= r[0] <= self.span[1]]
                rows = inside or rows
            if not rows:
                return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"]}
            reasons = {n for n, b in self.REASON_BITS.items() if any(r[2] & b for r in rows)}
            out = {"sm_mhz": statistics.median(r[1] for r in rows), "sm_mhz_min": min(r[1] for r in rows),
                   "sm_max_mhz": self.max_mhz, "samples": len(rows),
                   "power_w_max": round(max(r[3] for r in rows), 1),
                   "source": (f"NVML sampled continuously from the timed region's start to {int(self.TRAIL_S * 1e3)} "
                              "ms past its end (NVML refreshes every ~100 ms)") if self.span else "NVML"}
            if self.throttle_ms is not None:
                out["throttle_ms"] = self.throttle_ms
                out["region_ms"] = self.region_ms
                out["throttle_span_ms"] = self.throttle_span_ms  # covers the region, from just before it
                # a power-brake slowdown is one of the hardware slowdowns nvidia-smi reports as hw_slowdown
                reasons |= {"hw_slowdown" if n == "hw_power_brake_slowdown" else n
                            for n, v in self.throttle_ms.items() if v > 0}
            out["reasons"] = sorted(reasons)
            return out
        if self.proc is None or self.tmp is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.tmp.name) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 8 or (self.uuid and parts[0] != self.uuid):
                    continue
                rows.append(parts)
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": float(rows[0][2]),
                "samples": len(rows), "reasons": reasons, "source": "nvidia-smi every 200 ms"}


# ----------------------------------------------------------------------------------------- steps
def unit_plan(w: Workload, info: shard.RankInfo, scaling: str):
    """(heads of this rank, seed offset, layers per job) for weak / strong scaling."""
    if scaling == "weak":
        return range(w.H), info.rank, info.world
    return shard.unit_range(w.H, info.rank, info.world), 0, 1


def restrict_heads(w: Workload, heads: int) -> Workload:
    """The workload with only `heads` heads (profiling runs); 0 keeps it whole."""
    if heads <= 0 or heads >= w.H:
        return w
    from dataclasses import replace
    return replace(w, H=heads, name=f"{w.name}[{heads} heads]")


def make_step(w: Workload, api, fp8: bool = False):
    """Returns step(q, k, v, do, de) -> (out, grads) running forward + backward through `api`
    (fp8: VMonarch with e4m3 R-step operands, an option of this package only)."""
    if w.kind == "vmonarch":
        kw = {"fp8_r_step": True} if fp8 else {}

        def step(q, k, v, do, de):
            z = api.vmonarch_attention(q, k, v, w.m, w.b, w.iters, recompute_tokens=w.recompute, **kw)
            return z, torch.autograd.grad(z, (q, k, v), do)
    else:
        def step(q, k, v, do, de):
            o, e = api.flash_entropy_attention(q, k, v)
            return o, torch.autograd.grad((o, e), (q, k, v), (do, de))
    return step


def scaled_flops(w: Workload, n_heads: int) -> float:
    f = w.flops()
    return (f["fwd"] + f["bwd"]) * n_heads / w.H


def time_steps(step, args_dev, steps: int, warmup: int, device, launches=None, clock=None) -> float:
    """ms per step: W warm-up steps, then K steps bracketed by barrier + synchronize, CUDA events.
    `launches`, when given, is a list that receives this library's kernel launches issued by the
    K timed steps (warm-up excluded); `clock` (a ClockSampler) is given the timed region's host
    time span."""
    count = lambda: 0  # noqa: E731  (other arms load nothing of this library)
    if launches is not None:
        from vmonarch_b200 import ops
        count = ops.kernel_launches
    for _ in range(warmup):
        step(*args_dev)
    torch.cuda.synchronize(device)
    shard.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0 = count()
    if clock is not None:
        clock.begin()
    start.record()
    for _ in range(steps):
        step(*args_dev)
    end.record()
    n1 = count()
    torch.cuda.synchronize(device)
    if clock is not None:
        clock.end()
    shard.barrier()
    if launches is not None:
        launches.append(n1 - n0)
    return start.elapsed_time(end) / steps


def time_e2e(step, host, steps: int, device) -> float:
    """ms per step through the public API with host-resident inputs.

    Step t's inputs are copied host->device on a dedicated stream while step t-1 computes (two
    device buffer sets); every timed step's copy is issued inside the timed region (the first one
    waits for the start event). Each step's loss sum(out * dO) is copied back to pinned host
    memory, and the host reads the last one after the final synchronize. One warm-up step, then
    `steps` timed steps bracketed by barrier + synchronize."""
    comp = torch.cuda.current_stream(device)
    copy = torch.cuda.Stream(device)
    bufs = [[torch.empty_like(h, device=device) for h in host] for _ in range(2)]
    loss_host = torch.empty(steps + 1, dtype=torch.float32, pin_memory=True)
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    def issue_copy(t):
        b = t % 2
        with torch.cuda.stream(copy):
            if t >= 2:
                copy.wait_event(freed[b])
            for dst, src in zip(bufs[b], host):
                dst.copy_(src, non_blocking=True)
            copied[b].record(copy)

    def run(t):
        b = t % 2
        comp.wait_event(copied[b])
        leaves = [x.detach().requires_grad_() if i < 3 else x for i, x in enumerate(bufs[b])]
        out, grads = step(*leaves)
        loss = (out.float() * leaves[3].float()).sum()
        freed[b].record(comp)
        loss_host[t].copy_(loss, non_blocking=True)

    issue_copy(0)
    run(0)                                   # warm-up step
    torch.cuda.synchronize(device)
    shard.barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(comp)
    copy.wait_event(start)                   # step 1's copy starts inside the timed region
    issue_copy(1)
    for t in range(1, steps + 1):
        if t + 1 <= steps:
            issue_copy(t + 1)
        run(t)
    end.record(comp)
    torch.cuda.synchronize(device)
    shard.barrier()
    _ = float(loss_host[steps])              # the last step's result, read on the host
    return start.elapsed_time(end) / steps


def kernel_flops(name: str, a) -> tuple[float, float]:
    """(algorithmic FLOPs, algorithmic HBM bytes) of one C-ABI call, from its argument struct."""
    if name == "vmb_fea_fwd":
        f = 2.0 * a.batch * a.n_q * a.n_kv * (a.d + a.dv)
        by = 2.0 * a.batch * (a.n_q * (a.d + a.dv) + a.n_kv * (a.d + a.dv))
        return f, by
    if name == "vmb_fea_bwd":
        f = 2.0 * a.batch * a.n_q * a.n_kv * (3 * a.d + 2 * a.dv)
        by = 2.0 * a.batch * (a.n_q * (a.d + 2 * a.dv) + 2 * a.n_kv * (a.d + a.dv))
        return f, by
    dv = a.dw - a.d if a.last else a.d
    n = a.bh * a.m * a.b
    f = 2.0 * a.bh * a.b * a.m * a.m * (a.d + dv) * (2 if name == "vmb_lstep_bwd" else 1)
    by = n * (2 * a.d + 2 * a.dw + 4 + 2 * dv) if name == "vmb_lstep_fwd" else n * (2 * a.d + 4 * a.dw + 4 + 8 * a.d)
    return f, by


def call_key(name: str, a) -> str:
    """Entry point + shape: calls with the same key run the same kernels on the same sizes."""
    if name.startswith("vmb_fea"):
        return f"{name}[batch={a.batch},n_q={a.n_q},n_kv={a.n_kv},d={a.d},dv={a.dv}]"
    return f"{name}[bh={a.bh},m={a.m},b={a.b},d={a.d},dw={a.dw}]"


def profile_step(step, args_dev, device) -> dict:
    """One step with every C-ABI call bracketed by CUDA events on the current stream."""
    from vmonarch_b200 import ops
    recs = []

    @contextlib.contextmanager
    def timer(name, a):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        yield
        e.record()
        recs.append((call_key(name, a), kernel_flops(name, a), s, e))

    ops.set_timer(timer)
    try:
        step(*args_dev)
    finally:
        ops.set_timer(None)
    torch.cuda.synchronize(device)
    per = {}
    for key, (f, by), s, e in recs:
        d = per.setdefault(key, {"launches": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0})
        d["launches"] += 1
        d["ms"] += s.elapsed_time(e)
        d["flops"] += f
        d["bytes"] += by
    return per


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def roofline(per: dict) -> dict:
    """The dominant call group (entry point + shape) of one step, against the measured peak."""
    peaks, src = load_peaks()
    name, d = max(per.items(), key=lambda kv: kv[1]["ms"])
    total = sum(x["ms"] for x in per.values())
    if name.startswith("vmb_fea"):
        achieved = d["flops"] / (d["ms"] * 1e-3) / 1e12
        peak, unit, bound = peaks["bf16_tflops_sustained"], "TFLOP/s", "tensor"
        per_launch = d["flops"] / d["launches"]
    else:
        achieved = d["bytes"] / (d["ms"] * 1e-3) / 1e9
        peak, unit, bound = peaks["hbm_gbs"], "GB/s", "hbm"
        per_launch = d["bytes"] / d["launches"]
    traffic = None
    tp = ROOT / "profiles" / "traffic.txt"   # "<call key> <DRAM bytes per launch>" from an ncu capture
    if tp.exists():
        for line in tp.read_text().splitlines():
            parts = line.split()
            if len(parts) == 2 and parts[0] == name:
                traffic = float(parts[1])
    return {"kernel": name, "bound": bound, "achieved": round(achieved, 2), "peak": peak, "unit": unit,
            "frac": round(achieved / peak, 4), "peak_source": f"{src} (sustained bf16)" if bound == "tensor" else src,
            "per_launch_algorithmic": per_launch, "avg_launch_ms": round(d["ms"] / d["launches"], 4),
            "share_of_step": round(d["ms"] / total, 4), "traffic": traffic,
            "calls": {k: {"launches": v["launches"], "ms": round(v["ms"], 3)} for k, v in per.items()}}


# ----------------------------------------------------------------------------------------- CPU
def cpu_reference_sample(w: Workload, seed: int, budget_s: float, steps: int, warmup: int,
                         min_seconds: float = 0.0) -> dict:
    """The reference's CPU path (fp32 oracle) on whole heads of the workload; TFLOP/s of fwd+bwd.
    `warmup` untimed samples (at most one), then at least `steps` timed samples and at least
    `min_seconds` of timed work, stopping early only when `budget_s` of wall clock is spent."""
    import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    q, k, v, do, de = make_inputs(w, seed=seed, heads=range(0, 1), dtype=torch.float32)

    def one():
        leaves = [t.clone().requires_grad_() for t in (q, k, v)]
        if w.kind == "vmonarch":
            z = oracle.vmonarch_attention(*leaves, w.m, w.b, w.iters, recompute_tokens=w.recompute)
            torch.autograd.grad(z, leaves, do)
        else:
            o, e = oracle.entropy_attention(*leaves, w.D ** -0.5)
            torch.autograd.grad((o, e), leaves, (do, de))

    t0 = time.perf_counter()
    for _ in range(min(warmup, 1)):
        one()
    times = []
    while len(times) < max(steps, 1) or sum(times) < min_seconds:
        t = time.perf_counter()
        one()
        times.append(time.perf_counter() - t)
        if time.perf_counter() - t0 > budget_s:
            break
    sec = statistics.mean(times)
    return {"value": round(scaled_flops(w, 1) / sec / 1e12, 5), "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port", "seconds_per_sample": round(sec, 3), "timed_samples": len(times),
            "sample": f"1 of {w.H} heads of {w.name} (B=1,H=1,N={w.N}), fp32 forward+backward on the host, "
                      f"extrapolates x{w.H} per layer"}


# ----------------------------------------------------------------------------------------- arms
def capture_step(step, args_dev, warmup: int, device):
    """Captures one step in a CUDA graph after `warmup` eager steps on a side stream (the pattern
    torch documents for whole-network capture). Returns the graph, the outputs every replay
    rewrites, and the number of this library's kernels one replay launches."""
    from vmonarch_b200 import ops
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(max(warmup, 1)):
            step(*args_dev)
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    n0 = ops.kernel_launches()
    with torch.cuda.graph(graph):
        outs = step(*args_dev)
    return graph, outs, ops.kernel_launches() - n0


def l2_note(w: Workload) -> str:
    """How the timed steps relate to the 126 MB L2 (no flush is done between steps)."""
    q_bytes = w.B * w.H * w.N * w.D * 2
    if q_bytes > 126 * 2**20:
        return "inputs and activations larger than L2 (no flush needed)"
    return f"not flushed: q is {q_bytes / 2**20:.0f} MB, the step's working set may stay in L2 (small, launch-bound size)"


def data_note(w: Workload) -> str:
    if w.shared == "frame":
        return f"synthetic (seeded N(0,1) + per-frame shared mean, std {w.shared_std})"
    if w.shared == "block1024":
        return f"synthetic (seeded N(0,1) + per-1024-token-block shared component, std {w.shared_std})"
    return "synthetic (seeded N(0,1))"


def base_line(args, w, n_gpus, ms, value, impl=None) -> dict:
    """The contract's keys. `config` is built from the arguments alone, so both arms of one
    command line report the same config."""
    strong = args.scaling == "strong"
    per_rank = f"{-(-w.H // n_gpus)}" if w.H % n_gpus else f"{w.H // n_gpus}"
    line = {"metric": METRIC, "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": n_gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "bf16", "data": data_note(w),
            "config": {"workload": w.name, "B": w.B, "H": w.H, "num_blocks": w.m, "block_size": w.b, "N": w.N,
                       "D": w.D, "num_iters": w.iters, "recompute_tokens": w.recompute,
                       "layers_per_job": 1 if strong else n_gpus,
                       "parallelism": (f"heads split over {n_gpus} GPUs ({per_rank} per GPU), no collective on the "
                                       "hot path" if strong else f"one full layer per GPU x{n_gpus}, no collective"),
                       "l2": l2_note(w), "cuda_graph": bool(args.graph)}}
    if getattr(args, "fp8_r_step", False):
        line["config"]["r_step_operands"] = "e4m3 (fp8_r_step)"
    if impl:
        line["impl"] = impl
    return line


def verify_shards(w: Workload, step, dev, info, device, seed: int) -> dict:
    """Multi-GPU check, outside the timed region: one more step on every rank, an NCCL all_gather of
    z (or o) and the three input gradients of every head, then rank 0 runs two heads on its GPU
    alone (across the boundary between ranks 0 and 1 when N > 1) and compares. Heads are
    independent problems, but the kernels' work split depends on how many heads a call holds, so
    the comparison allows fp32-summation-order differences (1e-2 of max|ref| + 1e-3)."""
    out, grads = step(*dev)
    names = ("z" if w.kind == "vmonarch" else "o", "dq", "dk", "dv")
    # units on dim 0: (B, Hs, N, C) -> (Hs, B, N, C)
    local = [t.detach().transpose(0, 1).contiguous() for t in (out, *grads)]
    del out, grads
    full = [shard.gather_units(t, w.H, info.world) for t in local]
    del local
    res = {"gathered": list(names), "heads_gathered": w.H, "collective": "all_gather" if info.world > 1 else "none"}
    if info.rank == 0:
        h0 = max(shard.unit_range(w.H, 1, info.world).start - 1, 0) if info.world > 1 else 0
        h0 = min(h0, w.H - 2)
        q, k, v, do, de = make_inputs(w, seed=seed, heads=range(h0, h0 + 2))
        ref_dev = [t.to(device) for t in (q, k, v, do, de)]
        ref_dev = [t.requires_grad_() if i < 3 else t for i, t in enumerate(ref_dev)]
        r_out, r_grads = step(*ref_dev)
        ok, diffs = True, {}
        for n, got, want in zip(names, full, (r_out, *r_grads)):
            want = want.detach().transpose(0, 1).float()
            err = (got[h0:h0 + 2].float() - want).abs().max().item()
            tol = 1e-2 * want.abs().max().item() + 1e-3
            diffs[n] = round(err, 6)
            ok = ok and err <= tol and bool(torch.isfinite(got.float()).all())
        res.update({"heads_checked": [h0, h0 + 1], "max_abs_diff": diffs, "ok": ok,
                    "checksum_abs_sum": {n: round(t.float().abs().sum().item(), 3) for n, t in zip(names, full)}})
    del full
    shard.barrier()
    return res


def fea_forward_probe(args, device) -> dict:
    """FlashEntropyAttention forward at the fea32k configuration (B=1, H=24, N=32768, D=128; the
    configuration the forward-throughput target is quoted on): this library's forward and, when
    baseline/_ref holds the reference, the reference's Triton forward on the same inputs, each with
    3 warm-up calls (the reference autotunes on its first) and the mean of 10 timed calls (CUDA
    events on the current stream)."""
    import vmonarch_b200 as api
    w = WORKLOADS["fea32k"]
    q, k, v, _, _ = (t.to(device) for t in make_inputs(w, seed=args.seed))
    flops = w.flops()["fwd"]
    peaks, src = load_peaks()

    def timed(fn, n=10, warm=3):
        with torch.no_grad():
            for _ in range(warm):
                fn()
            torch.cuda.synchronize(device)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(n):
                fn()
            e.record()
            torch.cuda.synchronize(device)
        return s.elapsed_time(e) / n

    ms = timed(lambda: api.flash_entropy_attention(q, k, v))
    tf = flops / (ms * 1e-3) / 1e12
    res = {"workload": "fea32k forward (B=1, H=24, N=32768, D=Dv=128)", "flops": flops, "ms": round(ms, 4),
           "tflops": round(tf, 2), "frac_of_measured_burst": round(tf / peaks["bf16_tflops"], 4),
           "frac_of_nominal_2250": round(tf / 2250.0, 4), "peak_source": src}
    ref_dir = ROOT / "baseline" / "_ref"
    if (ref_dir / "video_monarch_attention").is_dir():
        sys.path.insert(0, str(ref_dir))
        try:
            import video_monarch_attention as ref
            rms = timed(lambda: ref.flash_entropy_attention(q, k, v))
            res["triton_reference_ms"] = round(rms, 4)
            res["triton_reference_tflops"] = round(flops / (rms * 1e-3) / 1e12, 2)
        except Exception as exc:  # pragma: no cover - depends on the box
            res["triton_reference"] = f"unavailable: {type(exc).__name__}: {str(exc).splitlines()[0][:160]}"
        finally:
            sys.path.remove(str(ref_dir))
    else:
        res["triton_reference"] = "unavailable: baseline/_ref does not hold the reference"
    del q, k, v
    return res


def run_ours(args, info, device):
    import vmonarch_b200 as api
    w = restrict_heads(WORKLOADS[args.workload], args.heads)
    heads, seed_off, layers = unit_plan(w, info, args.scaling)
    q, k, v, do, de = make_inputs(w, seed=args.seed + seed_off, heads=heads, pin=True)
    if w.kind == "vmonarch":
        de = de[..., :0]  # not an input of the VMonarch step: nothing to copy
    dev = [t.to(device, non_blocking=True) for t in (q, k, v, do, de)]
    dev = [t.requires_grad_() if i < 3 else t for i, t in enumerate(dev)]
    step = make_step(w, api, fp8=args.fp8_r_step)
    n_local = len(heads)
    flops_local = scaled_flops(w, n_local)
    flops_job = flops_local * (info.world if args.scaling == "weak" else 1)
    if args.scaling == "strong":
        flops_job = scaled_flops(w, w.H)

    if args.graph:
        graph, graph_outs, per_replay = capture_step(step, dev, args.warmup, device)
        with ClockSampler(device) as clk:
            ms = time_steps(lambda *_: graph.replay(), dev, args.steps, args.warmup, device, clock=clk)
        launches = per_replay * args.steps
        del graph, graph_outs
    else:
        counted = []
        with ClockSampler(device) as clk:
            ms = time_steps(step, dev, args.steps, args.warmup, device, launches=counted, clock=clk)
        launches = counted[0]
    ms_max = shard.max_over_ranks(ms, device)
    value = flops_job / (ms_max * 1e-3) / 1e12
    per = profile_step(step, dev, device)

    e2e = None
    if not args.no_e2e:
        # at least 10 steps: the pipeline's one unoverlapped compute (fill) is spread over the run
        n_e2e = max(args.steps, 10)
        ms_e2e = time_e2e(step, (q, k, v, do, de), n_e2e, device)
        ms_e2e = shard.max_over_ranks(ms_e2e, device)
        h2d = sum(t.numel() * t.element_size() for t in (q, k, v, do, de))
        h2d_job = h2d * info.world if args.scaling == "weak" else sum(
            t.numel() * t.element_size() // max(n_local, 1) * w.H for t in (q, k, v, do, de))
        e2e = {"value": round(flops_job / (ms_e2e * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
               "ms_per_step": round(ms_e2e, 3), "h2d_bytes_per_step": h2d_job, "d2h_bytes_per_step": 4 * info.world,
               "h2d_bytes_per_rank": h2d, "steps": n_e2e,
               "method": "every step copies its inputs (each rank its own heads) from pinned host memory (on a "
                         "copy stream, overlapping the previous step's compute, double-buffered) and reads its "
                         "loss back; the first step's copy and the last step's compute are inside the timed region"}

    verification = None
    if not args.no_verify and args.scaling == "strong" and w.H >= 2:
        verification = verify_shards(w, step, dev, info, device, args.seed)

    fea_fwd = None
    if info.world == 1 and not args.no_fea_forward:
        fea_fwd = fea_forward_probe(args, device)

    if info.rank != 0:
        return None
    line = base_line(args, w, info.world, ms_max, value)
    f = w.flops()
    line["dense_equivalent_tflops"] = round(3.5 * f["dense_fwd"] * n_local / w.H * layers / (ms_max * 1e-3) / 1e12, 2)
    line["flops_per_step"] = flops_job
    line["roofline"] = roofline(per)
    line["e2e"] = e2e
    line["gpu_launches"] = int(launches)
    line["clocks"] = clk.summary()
    if verification is not None:
        line["verification"] = verification
    if fea_fwd is not None:
        line["fea_forward"] = fea_fwd
    line["cpu_baseline"] = None
    if info.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_reference_sample(w, args.seed, 30.0, 3, 1, min_seconds=10.0)
    return line


def repo_libraries_mapped() -> list[str]:
    """Shared objects of this repository mapped into the process (Linux /proc/self/maps)."""
    try:
        maps = Path("/proc/self/maps").read_text()
    except OSError:
        return []
    root = str(ROOT)
    return sorted({ln.split()[-1] for ln in maps.splitlines() if ln.split() and ln.split()[-1].startswith(root)
                   and ".so" in ln.split()[-1]})


def run_reference(args, info):
    if info.rank != 0:
        return None
    w = WORKLOADS[args.workload]
    cpu = cpu_reference_sample(w, args.seed, args.cpu_budget_s, args.steps, args.warmup)
    ms = scaled_flops(w, w.H) / (cpu["value"] * 1e12) * 1e3  # one full layer, extrapolated from the heads
    line = base_line(args, w, info.world, ms, cpu["value"], impl="reference")
    line["value"] = cpu["value"]  # the same figure as cpu_baseline and e2e, not re-rounded
    line["steps"] = cpu["timed_samples"]
    line["cpu_baseline"] = cpu
    line["e2e"] = {"value": cpu["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    line["gpu_launches"] = 0
    line["repo_libraries_mapped"] = repo_libraries_mapped()
    return line


def run_triton(args, info, device):
    """The reference's own Triton path from baseline/_ref on the same GPU (comparison only).
    If its backward cannot launch on this GPU (the dit14b last R step needs more shared memory
    than a B200 has), or with --fwd-only, the forward alone is timed and the line says so."""
    ref_dir = ROOT / "baseline" / "_ref"
    sys.path.insert(0, str(ref_dir))
    try:
        import video_monarch_attention as ref
    except Exception as exc:  # pragma: no cover - depends on the box
        return {"impl": "reference-triton", "unavailable": f"cannot import the reference: {exc}"}
    w = WORKLOADS[args.workload]
    heads, seed_off, layers = unit_plan(w, info, args.scaling)
    q, k, v, do, de = make_inputs(w, seed=args.seed + seed_off, heads=heads)
    dev = [t.to(device) for t in (q, k, v, do, de)]
    dev = [t.requires_grad_() if i < 3 else t for i, t in enumerate(dev)]
    full = make_step(w, ref)
    mode, note = "forward+backward", None
    step = full
    if args.fwd_only:
        mode = "forward only"
    else:
        try:
            full(*dev)
            torch.cuda.synchronize(device)
        except Exception as exc:  # the reference's Triton backward may not fit this GPU
            note = f"reference backward failed on this GPU: {type(exc).__name__}: {str(exc).splitlines()[0][:160]}"
            mode = "forward only"
    if mode == "forward only":
        if w.kind == "vmonarch":
            def step(q, k, v, do, de):
                with torch.no_grad():
                    return ref.vmonarch_attention(q, k, v, w.m, w.b, w.iters, recompute_tokens=w.recompute)
        else:
            def step(q, k, v, do, de):
                with torch.no_grad():
                    return ref.flash_entropy_attention(q, k, v)
    with ClockSampler(device) as clk:
        ms = time_steps(step, dev, args.steps, args.warmup, device, clock=clk)
    ms_max = shard.max_over_ranks(ms, device)
    f = w.flops()
    per_head = (f["fwd"] + (f["bwd"] if mode == "forward+backward" else 0.0)) / w.H
    flops_job = per_head * len(heads) * (info.world if args.scaling == "weak" else 1)
    if args.scaling == "strong":
        flops_job = per_head * w.H
    if info.rank != 0:
        return None
    line = base_line(args, w, info.world, ms_max, flops_job / (ms_max * 1e-3) / 1e12, impl="reference-triton")
    line["mode"] = mode
    if note:
        line["note"] = note
    line["clocks"] = clk.summary()
    return line


def main():
    args = parse_args()
    info = shard.env_rank()
    if args.impl == "reference":
        line = run_reference(args, info)  # rank 0 only; no process group, the other ranks exit at once
    else:
        device = torch.device("cuda", info.local_rank)
        torch.cuda.set_device(device)
        shard.init("nccl")
        line = run_ours(args, info, device) if args.impl == "ours" else run_triton(args, info, device)
    if line is not None:
        print(json.dumps(line), flush=True)
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
