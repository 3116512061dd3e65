"""Benchmark of the B200 token sampler on BASELINE.json's headline metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2p] [--impl ours|reference]

One step = one rsc_sample call over a batch of logit rows already resident in
HBM (config cfg2p by default: 1024 rows x 151936 f32, T 0.8, top-k 40,
top-p 0.95, per-row uniforms). For N > 1 (torchrun, one rank per GPU) every
rank samples its own batch of the same shape (weak scaling, rows sharded with
no collective); the time is the max over ranks. Rank 0 prints one JSON line.

--config cfg4 with N > 1 runs the vocab-sharded mode instead: every rank holds
1/N of the columns of all 8192 rows, builds its shard records
(rsc_shard_partial), all-gathers them with NCCL over NVLink, and merges
(rsc_shard_merge); the job's rows are fixed (strong scaling).

`--impl reference` times the reference's CPU path instead: the C++
restatement of rusticide-sampling (oracle/, the reference's Rust cannot be
built on this image) on all host cores, on bounded samples of the same
workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_BYTES = 126 * 1024 * 1024

# The JSON line is the only output on stdout. Everything else written to file
# descriptor 1, by Python or by native libraries (NCCL prints its version there
# on some systems), goes to stderr; emit() writes to the original stdout.
_JSON_FD = None


def claim_stdout() -> None:
    global _JSON_FD
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)


def emit(line: dict) -> None:
    data = (json.dumps(line) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, data)


def env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def committed_traffic(config: str) -> float | None:
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary of this workload (profiles/), or None."""
    p = ROOT / "profiles" / f"stream_topk_{config}.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock and throttle-reason samples while the benchmark runs;
    `stop(window)` keeps the samples taken inside the timed region."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.tmp = None

    def start(self):
        try:
            self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "50"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    @staticmethod
    def _when(stamp: str):
        from datetime import datetime
        for fmt in ("%Y/%m/%d %H:%M:%S.%f", "%Y/%m/%d %H:%M:%S"):
            try:
                return datetime.strptime(stamp, fmt).timestamp()
            except ValueError:
                pass
        return None

    def stop(self, window=None) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.tmp.flush()
        rows = []
        for line in Path(self.tmp.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10:
                rows.append(parts)
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        scope = "whole run"
        if window is not None:
            inside = [r for r in rows
                      if (w := self._when(r[0])) is not None and window[0] <= w <= window[1]]
            if inside:
                rows, scope = inside, "timed region"

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None

        sm = [num(r[2]) for r in rows if num(r[2]) is not None]
        mx = [num(r[3]) for r in rows if num(r[3]) is not None]
        pw = [num(r[4]) for r in rows if num(r[4]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for name, val in zip(names, r[6:10]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "power_w": statistics.median(pw) if pw else None,
                "reasons": sorted(reasons), "samples": len(rows), "scope": scope}


def device_logits(cfg, rows: int, seed: int, device):
    """The config's distribution, generated on the device from a seed."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    scale = 2.0 if cfg.dist == "peaked" else 0.5
    x = torch.randn(rows, cfg.vocab, device=device, generator=g) * scale
    lo, hi = cfg.spikes
    if hi > 0:
        n = torch.randint(lo, hi + 1, (rows, 1), device=device, generator=g)
        idx = torch.randint(0, cfg.vocab, (rows, hi), device=device, generator=g)
        boost = 5.0 + 7.0 * torch.rand(rows, hi, device=device, generator=g)
        boost = boost * (torch.arange(hi, device=device).unsqueeze(0) < n)
        x.scatter_add_(1, idx, boost)
    u = torch.rand(rows, device=device, generator=g)
    return x.contiguous(), u


def cpu_baseline(x_host, u_host, params, seconds: float, threads: int, greedy: bool = False) -> dict:
    """The oracle (C++ restatement of the reference) on the host cores, on
    repeated passes over a sample of the rows, for about `seconds`."""
    from oracle import oracle as O
    op = O.params(params.temperature, params.top_k, params.top_p)
    rows = 0
    t0 = time.perf_counter()
    while True:
        if greedy:
            O.greedy_rows(x_host, threads=threads)
        else:
            O.sample_rows(x_host, op, u_host, threads=threads)
        rows += x_host.shape[0]
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    # The same on one core (the reference samples one row per call on one
    # thread): the first rows of the sample, for a quarter of the time.
    n1 = max(1, x_host.shape[0] // max(threads, 1))
    x1, u1 = x_host[:n1], u_host[:n1]
    rows1 = 0
    t1 = time.perf_counter()
    while True:
        if greedy:
            O.greedy_rows(x1, threads=1)
        else:
            O.sample_rows(x1, op, u1, threads=1)
        rows1 += n1
        if time.perf_counter() - t1 >= seconds / 4:
            break
    dt1 = time.perf_counter() - t1
    return {"value": rows / dt, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{x_host.shape[0]} rows x {x_host.shape[1]} of the workload, "
                      f"{rows // x_host.shape[0]} passes, {dt:.1f} s, {threads} threads",
            "single_core_value": rows1 / dt1,
            "single_core_sample": f"{n1} rows, {rows1 // n1} passes, {dt1:.1f} s, 1 thread"}


def run_reference(args, cfg, rank: int, world: int) -> None:
    if rank != 0:
        return
    import numpy as np
    from rusticide_b200 import SamplingParams, synth
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    sample_rows = max(threads * 4, 64)
    x = synth.make_config(cfg, rows=sample_rows, base_seed=1234)
    u = synth.uniforms(sample_rows, seed=99)
    params = SamplingParams(cfg.temperature, cfg.top_k, cfg.top_p)
    op = O.params(cfg.temperature, cfg.top_k, cfg.top_p)

    def ref_step():
        if cfg.greedy:
            O.greedy_rows(x, threads=threads)
        else:
            O.sample_rows(x, op, u, threads=threads)

    # Bound the whole run to about `ref_seconds`: shrink the per-step sample
    # (down to one row per thread) when K steps of the first size would not fit.
    t_w = time.perf_counter()
    ref_step()
    per_step = time.perf_counter() - t_w
    budget = args.ref_seconds / max(args.steps + args.warmup, 1)
    if per_step > budget:
        sample_rows = max(threads, int(sample_rows * budget / per_step))
        sample_rows = min(sample_rows, x.shape[0])
        x, u = np.ascontiguousarray(x[:sample_rows]), np.ascontiguousarray(u[:sample_rows])
    for _ in range(args.warmup):
        ref_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ref_step()
    dt = time.perf_counter() - t0
    value = sample_rows * args.steps / dt
    line = {
        "impl": "reference",
        "metric": "sampled rows/sec",
        "value": value,
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1000 / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": cfg.name, "rows": cfg.rows, "vocab": cfg.vocab,
                   "temperature": cfg.temperature, "top_k": cfg.top_k, "top_p": cfg.top_p,
                   "step_sample_rows": sample_rows},
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "sample": f"{sample_rows} rows x {cfg.vocab} per step"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference = C++ restatement of rusticide-sampling (Rust toolchain absent on this image)",
    }
    emit(line)


def main() -> None:
    claim_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="cfg2p")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=150.0,
                    help="bound on the reference arm's run time")
    ap.add_argument("--rows", type=int, default=0,
                    help="rows per GPU (default: the config's); for small profiling captures")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)

    from rusticide_b200 import synth
    cfg = synth.CONFIGS[args.config]

    if args.impl == "reference":
        run_reference(args, cfg, rank, world)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from rusticide_b200 import SamplingParams, engine
    from rusticide_b200.sharding import VocabShardedSampler

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=device)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    params = SamplingParams(cfg.temperature, cfg.top_k, cfg.top_p)
    rows, vocab = (args.rows or cfg.rows), cfg.vocab
    sharded = cfg.name == "cfg4" and world > 1
    eng = engine(local)
    if sharded:
        # This rank's columns of every row (spikes spread over the shards),
        # and the same per-row uniforms on every rank: the merge must draw
        # identically everywhere.
        vs = VocabShardedSampler(eng, vocab)
        spk = max(1, cfg.spikes[0] // world)
        x, _ = device_logits(synth.Config(cfg.name, rows, vs.width, cfg.temperature, cfg.top_k,
                                          cfg.top_p, cfg.dist, (spk, spk)),
                             rows, 1234 + 7919 * rank, device)
        g = torch.Generator(device=device).manual_seed(4321)
        u = torch.rand(rows, device=device, generator=g)
        eng.ensure(rows, vs.width)
    else:
        x, u = device_logits(cfg, rows, 1234 + 7919 * rank, device)
        eng.ensure(rows, vocab)
    outs = eng._outputs(rows, True)
    stream = torch.cuda.current_stream(device)

    def step():
        if sharded:
            vs.sample(x, params, uniforms=u, out=outs)
        elif cfg.greedy:
            eng.greedy(x, out=outs)
        else:
            eng.sample(x, params, uniforms=u, out=outs)

    clocks = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                          if os.environ.get("CUDA_VISIBLE_DEVICES") else local)
    clocks.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    barrier()
    torch.cuda.synchronize(device)

    launches0 = eng.launch_count()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(device)
    wall1 = time.time()
    barrier()
    torch.cuda.synchronize(device)
    launches = eng.launch_count() - launches0
    t_ms = ev0.elapsed_time(ev1)

    # Per-call kernel time (every call bracketed by its own events).
    per = []
    for _ in range(min(args.steps, 50)):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step()
        b.record(stream)
        per.append((a, b))
    torch.cuda.synchronize(device)
    clk = clocks.stop((wall0, wall1))
    call_ms = statistics.mean(a.elapsed_time(b) for a, b in per)

    # End to end through the host-buffer entry point: H2D of the logits and
    # uniforms, sampling, D2H of ids, statuses and probabilities, every step.
    e2e_rows = rows
    if sharded:
        # The host-buffer entry point samples whole rows; the sharded job's
        # end-to-end figure is the device-resident step plus the copies of
        # this rank's shard in and the results out.
        x_host = torch.empty(x.shape, dtype=torch.float32, pin_memory=True)
        x_host.copy_(x)
        res_host = torch.empty(rows * 3, dtype=torch.int32, pin_memory=True)
        torch.cuda.synchronize(device)
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            x.copy_(x_host, non_blocking=True)
            step()
            res_host[:rows].copy_(outs[0], non_blocking=True)
            res_host[rows:2 * rows].copy_(outs[1], non_blocking=True)
            res_host[2 * rows:].copy_(outs[2].view(torch.int32), non_blocking=True)
            torch.cuda.synchronize(device)
        e2e_s = time.perf_counter() - t0
        barrier()
    else:
        x_host = torch.empty((rows, vocab), dtype=torch.float32, pin_memory=True)
        x_host.copy_(x)
        u_host = torch.empty(rows, dtype=torch.float32, pin_memory=True)
        u_host.copy_(u)
        xh, uh = x_host.numpy(), u_host.numpy()
        eng.pick_host(xh, params, None if cfg.greedy else uh)  # warm
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            eng.pick_host(xh, params, None if cfg.greedy else uh)
        e2e_s = time.perf_counter() - t0
        barrier()

    t_max = t_ms
    e2e_max = e2e_s
    if world > 1:
        tt = torch.tensor([t_ms, e2e_s], dtype=torch.float64, device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_max, e2e_max = float(tt[0]), float(tt[1])

    cpu = None
    if rank == 0 and world == 1:
        n_cpu = min(rows, 256)
        if cfg.greedy:
            params_cpu = SamplingParams(0.0, cfg.top_k, cfg.top_p)
        else:
            params_cpu = params
        cpu = cpu_baseline(x[:n_cpu].cpu().numpy(), u[:n_cpu].cpu().numpy(), params_cpu,
                           args.cpu_seconds, os.cpu_count() or 1, cfg.greedy)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return

    job_rows = rows if sharded else rows * world
    total_rows = job_rows * args.steps
    value = total_rows / (t_max / 1000.0)
    peak, peak_kind = measured_peak()
    alg_bytes = rows * (x.shape[1] if sharded else vocab) * 4
    # The dominant kernel's average duration per launch over the timed region
    # (this rank's CUDA events on the launching stream). One streaming launch
    # per step on the sampling path; consecutive launches overlap by
    # programmatic dependent launch, so this is the steady-state cost.
    launches_per_step = launches / args.steps if args.steps else 0
    step_s = t_ms / 1000.0 / args.steps
    achieved = alg_bytes / step_s / 1e9
    single = alg_bytes / (call_ms / 1000.0) / 1e9
    traffic = committed_traffic(args.config)
    line = {
        "metric": "sampled rows/sec",
        "value": value,
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": t_max / args.steps,
        "higher_is_better": True,
        "scaling": "strong" if sharded else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": cfg.name, "rows_per_gpu": rows, "vocab": vocab,
                   "temperature": cfg.temperature, "top_k": cfg.top_k, "top_p": cfg.top_p,
                   "mode": "greedy" if cfg.greedy else "sample_logits",
                   "parallelism": (f"vocab-sharded x{world} (NCCL all-gather of shard records)"
                                   if sharded else f"row-sharded x{world}"),
                   "l2": f"inputs {alg_bytes / 2**20:.0f} MiB > 126 MiB L2 (no flush needed)"},
        "hbm_gbs": achieved,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "launches_per_step": launches_per_step,
                     "single_call_gbs": single,
                     "single_call_us": call_ms * 1000.0,
                     "note": ("achieved = rows*vocab*4 B per step / CUDA-event time per step over "
                              "the timed region; single_call_* = one call bracketed by its own "
                              "events (no overlap with the next call)")},
        "e2e": {"value": job_rows * args.e2e_steps / e2e_max, "unit": "rows/s",
                "h2d_bytes_per_step": (rows * x.shape[1] * 4 if sharded else
                                       rows * vocab * 4 + (0 if cfg.greedy else rows * 4)),
                "d2h_bytes_per_step": rows * 12},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    emit(line)


if __name__ == "__main__":
    main()
