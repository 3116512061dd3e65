"""Benchmark of the B200 token sampler on BASELINE.json's headline metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2p] [--impl ours|reference]

One step = one rsc_sample call over a batch of logit rows already resident in
HBM (config cfg2p by default: 1024 rows x 151936 f32, T 0.8, top-k 40,
top-p 0.95, per-row uniforms). For N > 1 (torchrun, one rank per GPU) every
rank samples its own batch of the same shape (weak scaling, rows sharded with
no collective); the time is the max over ranks. Rank 0 prints one JSON line.

Besides the timed steps, the line carries:
  - `sustained`: the same step repeated for about a second, with the clocks
    sampled while it runs (the K-step region is shorter than nvidia-smi's
    50 ms sampling period at the driver's K);
  - `parity`: the per-config correctness counters, from the GPU's results on a
    256-row sample of the workload checked against the CPU oracle (outside
    every timed region);
  - `vocab_sharded`: config 4 (8192 x 151936, T 0.8, k 40, p 0.95) with the
    vocabulary split over the N ranks (rsc_shard_partial, an NCCL all-gather
    of the shard records, rsc_shard_merge), timed as the max over ranks and
    checked bit for bit against the unsharded call on the same rows; at N = 1
    the unsharded call alone, the strong-scaling base.

--config cfg4 with N > 1 makes the vocab-sharded mode the main step.
--config lmhead times the LM-head paths instead (a table, not the contract).

`--impl reference` times the reference's CPU path instead: the C++
restatement of rusticide-sampling (oracle/, the reference's Rust cannot be
built on this image) on all host cores, on the same 256-row sample the
cpu_baseline leg uses.
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
SAMPLE_ROWS = 256          # rows of the CPU sample (cpu_baseline, reference arm, parity)
SAMPLE_SEED = 1234         # synth row seeds SAMPLE_SEED + r
SAMPLE_USEED = 99          # synth.uniforms seed of the sample

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
    for name in (f"stream_topk_{config}.md", f"large_kernel_{config}.md"):
        p = ROOT / "profiles" / name
        if not p.exists():
            continue
        for line in p.read_text().splitlines():
            if line.startswith("dram_bytes_per_launch:"):
                try:
                    return float(line.split(":", 1)[1].split()[0])
                except ValueError:
                    return None
    return None


class ClockSampler:
    """nvidia-smi clock and throttle-reason samples while the benchmark runs;
    `stop(windows)` keeps the samples taken inside the first window that has
    any, and says which."""

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

    def stop(self, windows=()) -> dict:
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
        for name, (a, b) in windows:
            inside = [r for r in rows if (w := self._when(r[0])) is not None and a <= w <= b]
            if inside:
                rows, scope = inside, name
                break

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


def device_logits(cfg, rows: int, seed: int, device, vocab: int | None = None):
    """The config's distribution, generated on the device from a seed."""
    import torch
    vocab = vocab or cfg.vocab
    g = torch.Generator(device=device).manual_seed(seed)
    scale = 2.0 if cfg.dist == "peaked" else 0.5
    x = torch.randn(rows, vocab, device=device, generator=g) * scale
    lo, hi = cfg.spikes
    if hi > 0:
        n = torch.randint(lo, hi + 1, (rows, 1), device=device, generator=g)
        idx = torch.randint(0, vocab, (rows, hi), device=device, generator=g)
        boost = 5.0 + 7.0 * torch.rand(rows, hi, device=device, generator=g)
        boost = boost * (torch.arange(hi, device=device).unsqueeze(0) < n)
        x.scatter_add_(1, idx, boost)
    u = torch.rand(rows, device=device, generator=g)
    return x.contiguous(), u


def cpu_sample(cfg, rows: int = SAMPLE_ROWS):
    """The CPU sample of the workload: rows 0..rows-1 of the config's synthetic
    generator (numpy, seeds SAMPLE_SEED + r) and their uniforms. The same rows
    feed cpu_baseline, the reference arm and the parity counters."""
    from rusticide_b200 import synth
    rows = min(rows, cfg.rows)
    return synth.make_config(cfg, rows=rows, base_seed=SAMPLE_SEED), synth.uniforms(rows, SAMPLE_USEED)


def cpu_baseline(x_host, u_host, params, seconds: float, threads: int, greedy: bool = False) -> dict:
    """The oracle (C++ restatement of the reference) on the host cores, on
    repeated passes over a sample of the rows, for about `seconds`."""
    from oracle import oracle as O
    op = O.params(params.temperature, params.top_k, params.top_p)
    rows = 0

    def once(x, u, th):
        if greedy:
            O.greedy_rows(x, threads=th)
        else:
            O.sample_rows(x, op, u, threads=th)

    once(x_host[:threads], u_host[:threads], threads)  # starts the worker pool
    t0 = time.perf_counter()
    while True:
        once(x_host, u_host, threads)
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
        once(x1, u1, 1)
        rows1 += n1
        if time.perf_counter() - t1 >= seconds / 4:
            break
    dt1 = time.perf_counter() - t1
    return {"value": rows / dt, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{x_host.shape[0]} rows x {x_host.shape[1]} of the workload "
                      f"(synthetic seeds {SAMPLE_SEED}+r), {rows // x_host.shape[0]} passes, "
                      f"{dt:.1f} s, {threads} threads of a persistent pool",
            "single_core_value": rows1 / dt1,
            "single_core_sample": f"{n1} rows, {rows1 // n1} passes, {dt1:.1f} s, 1 thread"}


def workload_config(cfg, rows: int, world: int, sharded: bool) -> dict:
    return {"workload": cfg.name, "rows_per_gpu": rows, "vocab": cfg.vocab,
            "temperature": cfg.temperature, "top_k": cfg.top_k, "top_p": cfg.top_p,
            "mode": "greedy" if cfg.greedy else "sample_logits",
            "parallelism": (f"vocab-sharded x{world} (NCCL all-gather of shard records)"
                            if sharded else f"row-sharded x{world}"),
            "l2": f"inputs {rows * cfg.vocab * 4 / 2**20:.0f} MiB per GPU vs 126 MiB L2 "
                  f"({'no flush needed' if rows * cfg.vocab * 4 > L2_BYTES else 'L2-resident'})"}


def run_reference(args, cfg, rank: int, world: int) -> None:
    if rank != 0:
        return
    import numpy as np
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    x, u = cpu_sample(cfg)
    sample_rows = x.shape[0]
    op = O.params(cfg.temperature, cfg.top_k, cfg.top_p)

    def ref_step(xx, uu):
        if cfg.greedy:
            O.greedy_rows(xx, threads=threads)
        else:
            O.sample_rows(xx, op, uu, threads=threads)

    # Bound the whole run to about `ref_seconds`: shrink the per-step sample
    # (down to one row per thread) only when K steps of the full sample would
    # not fit.
    ref_step(x[:threads], u[:threads])  # starts the worker pool
    t_w = time.perf_counter()
    ref_step(x, u)
    per_step = time.perf_counter() - t_w
    budget = args.ref_seconds / max(args.steps + args.warmup, 1)
    if per_step > budget:
        sample_rows = min(x.shape[0], max(threads, int(sample_rows * budget / per_step)))
        x, u = np.ascontiguousarray(x[:sample_rows]), np.ascontiguousarray(u[:sample_rows])
    for _ in range(args.warmup):
        ref_step(x, u)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        ref_step(x, u)
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
        "config": workload_config(cfg, args.rows or cfg.rows, world, False),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": threads, "kind": "port",
                         "sample": f"{sample_rows} rows x {cfg.vocab} per step (synthetic seeds "
                                   f"{SAMPLE_SEED}+r, the cpu_baseline leg's sample), "
                                   f"{threads} threads of a persistent pool"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference = C++ restatement of rusticide-sampling (Rust toolchain absent on this image)",
    }
    emit(line)


def parity_counters(eng, cfg, params, device) -> dict:
    """The correctness counters of the workload's parameters (checked outside
    every timed region): the GPU samples the CPU sample's rows as one batch,
    and the oracle samples the same rows with the same uniforms.

      greedy_id_mismatches       rsc_greedy vs greedy_logits (must be 0)
      topk_set_mismatches        rows whose top-k survivor set differs (0)
      topp_set_mismatches        rows whose final survivor set differs (0)
      max_rel_prob_error         over every survivor's probability (<= 1e-5)
      sampled_id_mismatches      split into boundary (|u - CDF edge| < 1e-6)
                                 and non_boundary (must be 0)
      status_mismatches          per-row outcome codes (0)
      boundary_draws             rows whose u lies within 1e-6 of a CDF edge
      topp_boundary_cases        rows whose top-p running sum lies within 1e-6
                                 of p at the cut
    """
    import numpy as np
    import torch

    from oracle import oracle as O
    from rusticide_b200 import SamplingParams

    x_host, u_host = cpu_sample(cfg)
    rows, vocab = x_host.shape
    threads = os.cpu_count() or 1
    x = torch.from_numpy(x_host).to(device)
    u = torch.from_numpy(u_host).to(device)
    out = {"rows_checked": rows, "vocab": vocab, "sample": f"synthetic seeds {SAMPLE_SEED}+r"}

    gids, gst = eng.greedy(x)
    gw = O.greedy_rows(x_host, threads=threads)
    torch.cuda.synchronize(device)
    gids = gids.cpu().numpy().view(np.uint32)
    out["greedy_id_mismatches"] = int(np.sum((gids != gw["token"]) |
                                             ((gst.cpu().numpy() & 0xFF) != gw["status"])))
    if cfg.greedy:
        return out

    op = O.params(params.temperature, params.top_k, params.top_p)
    want = O.sample_rows(x_host, op, u_host, threads=threads)
    cap = vocab
    ids, st, probs, nsurv, surv, survp = eng.sample_ex(x, params, uniforms=u, survivor_cap=cap)
    p_k = SamplingParams(params.temperature, params.top_k, 1.0)
    _, _, _, nk, survk, _ = eng.sample_ex(x, p_k, uniforms=u, survivor_cap=cap)
    torch.cuda.synchronize(device)
    ids = ids.cpu().numpy().view(np.uint32)
    st = st.cpu().numpy()
    probs = probs.cpu().numpy()
    nsurv, surv, survp = nsurv.cpu().numpy(), surv.cpu().numpy(), survp.cpu().numpy()
    nk, survk = nk.cpu().numpy(), survk.cpu().numpy()
    opk = O.params(params.temperature, params.top_k, 1.0)

    topk_bad = topp_bad = 0
    max_rel = 0.0
    topp_edge = 0
    for r in range(rows):
        kidx, _ = O.filter_(x_host[r], opk)
        if nk[r] != len(kidx) or not np.array_equal(survk[r, :len(kidx)].view(np.uint32), kidx):
            topk_bad += 1
        pidx, pval = O.filter_(x_host[r], op)
        if nsurv[r] != len(pidx) or not np.array_equal(surv[r, :len(pidx)].view(np.uint32), pidx):
            topp_bad += 1
            continue
        if len(pidx):
            pw = O.softmax(pval)
            pg = survp[r, :len(pidx)]
            with np.errstate(divide="ignore", invalid="ignore"):
                rel = np.abs(pg.astype(np.float64) - pw) / np.abs(pw.astype(np.float64))
            rel = rel[np.isfinite(rel)]
            if rel.size:
                max_rel = max(max_rel, float(rel.max()))
        if params.top_p < 1.0:
            _, before, after = O.topp_edge(x_host[r], op)
            if min(abs(before - params.top_p), abs(after - params.top_p)) < 1e-6:
                topp_edge += 1
    near = (np.abs(u_host - want["cdf_lo"]) < 1e-6) | (np.abs(u_host - want["cdf_hi"]) < 1e-6)
    near &= want["consumed_draw"] != 0
    bad = ids != want["token"]
    with np.errstate(divide="ignore", invalid="ignore"):
        prel = np.abs(probs.astype(np.float64) - want["prob"]) / np.abs(want["prob"].astype(np.float64))
    prel = prel[np.isfinite(prel)]
    if prel.size:
        max_rel = max(max_rel, float(prel.max()))
    out.update({
        "topk_set_mismatches": int(topk_bad),
        "topp_set_mismatches": int(topp_bad),
        "max_rel_prob_error": max_rel,
        "sampled_id_mismatches": {"boundary": int(np.sum(bad & near)),
                                  "non_boundary": int(np.sum(bad & ~near))},
        "status_mismatches": int(np.sum((st & 0xFF) != want["status"])),
        "boundary_draws": int(np.sum(near)),
        "topp_boundary_cases": int(topp_edge),
    })
    return out


def vocab_sharded_leg(eng, world: int, rank: int, local: int, device, steps: int, warmup: int,
                      peak: float) -> dict | None:
    """Config 4 with the vocabulary split over the ranks, against the unsharded
    call on the same rows (see the module docstring). Every rank takes the
    same collective steps."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from oracle import oracle as O
    from rusticide_b200 import SamplingParams, synth
    from rusticide_b200.sharding import VocabShardedSampler

    cfg = synth.CONFIGS["cfg4"]
    rows, vocab = cfg.rows, cfg.vocab
    params = SamplingParams(cfg.temperature, cfg.top_k, cfg.top_p)
    full, u = device_logits(cfg, rows, 4242, device)
    if world > 1:
        # The same rows on every rank: rank 0's, broadcast over NVLink.
        dist.broadcast(full, 0)
        dist.broadcast(u, 0)
    eng.ensure(rows, vocab)
    stream = torch.cuda.current_stream(device)

    def timed(fn, n):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier(device_ids=[local])
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) * 1000.0 / n

    base = eng._outputs(rows, True)
    t_unsharded = timed(lambda: eng.sample(full, params, uniforms=u, out=base), steps)
    eng.sample(full, params, uniforms=u, out=base)
    res = {"config": "cfg4", "rows": rows, "vocab": vocab, "n_shards": world,
           "us_per_step_unsharded_1gpu": t_unsharded,
           "unsharded_gbs": rows * vocab * 4 / (t_unsharded * 1e-6) / 1e9}
    if world > 1:
        vs = VocabShardedSampler(eng, vocab)
        view = full[:, vs.offset:vs.offset + vs.width]
        outs = eng._outputs(rows, True)
        t = timed(lambda: vs.sample(view, params, uniforms=u, out=outs), steps)
        vs.sample(view, params, uniforms=u, out=outs)
        torch.cuda.synchronize(device)
        # The step's three parts timed apart (same buffers, every rank).
        records, gathered = vs._buffers(rows, params.top_k, device)
        t_part = timed(lambda: eng.shard_partial(view, vs.offset, vocab, params, records=records),
                       steps)
        t_gather = timed(lambda: dist.all_gather_into_tensor(gathered, records), steps)
        t_merge = timed(lambda: eng.shard_merge(gathered, world, rows, vocab, params, uniforms=u,
                                                out=outs), steps)
        vs.sample(view, params, uniforms=u, out=outs)
        torch.cuda.synchronize(device)
        same = (torch.equal(outs[0], base[0]) and torch.equal(outs[1], base[1])
                and torch.equal(outs[2].view(torch.int32), base[2].view(torch.int32)))
        stat = torch.tensor([t, 0.0 if same else 1.0, float(vs.width), t_part, t_gather, t_merge],
                            dtype=torch.float64, device=device)
        dist.all_reduce(stat, op=dist.ReduceOp.MAX)
        t_max, any_diff, wmax = float(stat[0]), float(stat[1]), float(stat[2])
        parts = {"partial_us": float(stat[3]), "allgather_us": float(stat[4]),
                 "merge_us": float(stat[5])}
        per_gpu_bytes = rows * wmax * 4
        res.update({
            "us_per_step": t_max,
            "shard_width_max": int(wmax),
            "per_gpu_gbs": per_gpu_bytes / (t_max * 1e-6) / 1e9,
            "per_gpu_frac": per_gpu_bytes / (t_max * 1e-6) / 1e9 / peak,
            "strong_scaling_eff": t_unsharded / (world * t_max),
            "bit_exact_vs_unsharded": any_diff == 0.0,
            "parts_max_over_ranks": parts,
            "note": "us_per_step = partial + NCCL all-gather + merge, max over ranks; "
                    "strong_scaling_eff = unsharded 1-GPU time / (N x sharded time)",
        })
        # The same step with the records read in place over NVLink (peer
        # memory) instead of all-gathered by NCCL.
        from rusticide_b200.sharding import PeerVocabShardedSampler
        pvs = PeerVocabShardedSampler(eng, vocab)
        pouts = eng._outputs(rows, True)
        t_peer = timed(lambda: pvs.sample(view, params, uniforms=u, out=pouts), steps)
        pvs.sample(view, params, uniforms=u, out=pouts)
        torch.cuda.synchronize(device)
        psame = (torch.equal(pouts[0], base[0]) and torch.equal(pouts[1], base[1])
                 and torch.equal(pouts[2].view(torch.int32), base[2].view(torch.int32)))
        pstat = torch.tensor([t_peer, 0.0 if psame else 1.0], dtype=torch.float64, device=device)
        dist.all_reduce(pstat, op=dist.ReduceOp.MAX)
        dist.barrier(device_ids=[local])
        res["peer_exchange"] = {
            "us_per_step": float(pstat[0]),
            "strong_scaling_eff": t_unsharded / (world * float(pstat[0])),
            "bit_exact_vs_unsharded": float(pstat[1]) == 0.0,
            "note": "partial + publish + merge reading every rank's records over NVLink "
                    "(rsc_shard_merge_peers), max over ranks"}
        del pvs
        got = outs
    else:
        res["us_per_step"] = t_unsharded
        got = base
    if rank == 0:
        n = 32
        xs = full[:n].cpu().numpy()
        us = u[:n].cpu().numpy()
        want = O.sample_rows(xs, O.params(cfg.temperature, cfg.top_k, cfg.top_p), us,
                             threads=os.cpu_count() or 1)
        gi = got[0][:n].cpu().numpy().view(np.uint32)
        gs = got[1][:n].cpu().numpy() & 0xFF
        res["oracle_rows_checked"] = n
        res["oracle_mismatches"] = int(np.sum((gi != want["token"]) | (gs != want["status"])))
    return res


def emulated_shards(args) -> None:
    """--config cfg4 --emulate-shards N on one GPU: the vocab-sharded step of
    one rank at N GPUs, with the shards emulated on this GPU. Times one
    rank's partial pass over its V/N columns (rsc_shard_partial), the merge of
    N records (rsc_shard_merge) and the unsharded call on the same rows, and
    checks the merged result bit for bit against the unsharded one. No
    collective runs: the all-gather of the records is a concatenation here."""
    import torch

    from rusticide_b200 import SamplingParams, engine, synth

    cfg = synth.CONFIGS["cfg4"]
    n = args.emulate_shards
    rows, vocab = (args.rows or cfg.rows), cfg.vocab
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    eng = engine(0)
    params = SamplingParams(cfg.temperature, cfg.top_k, cfg.top_p)
    x, u = device_logits(cfg, rows, 4242, device)
    eng.ensure(rows, vocab)
    bounds = [vocab * s // n for s in range(n + 1)]
    rb = eng.shard_record_bytes(params.top_k)
    gathered = torch.empty(n * rows * rb, dtype=torch.uint8, device=device)
    recs = [gathered[s * rows * rb:(s + 1) * rows * rb] for s in range(n)]
    outs = eng._outputs(rows, True)
    base = eng._outputs(rows, True)
    stream = torch.cuda.current_stream(device)

    def timed(fn, k):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(device)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(k):
            fn()
        b.record(stream)
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) * 1000.0 / k

    def partials():
        for s in range(n):
            eng.shard_partial(x[:, bounds[s]:bounds[s + 1]], bounds[s], vocab, params, records=recs[s])

    def merge():
        eng.shard_merge(gathered, n, rows, vocab, params, uniforms=u, out=outs)

    steps = max(args.steps, 1)
    t_unsharded = timed(lambda: eng.sample(x, params, uniforms=u, out=base), steps)
    t_one = timed(lambda: eng.shard_partial(x[:, bounds[0]:bounds[1]], bounds[0], vocab, params,
                                            records=recs[0]), steps)
    partials()
    t_merge = timed(merge, steps)
    merge()
    torch.cuda.synchronize(device)
    same = (torch.equal(outs[0], base[0]) and torch.equal(outs[1], base[1])
            and torch.equal(outs[2].view(torch.int32), base[2].view(torch.int32)))
    peak, _ = measured_peak()
    width = bounds[1] - bounds[0]
    emit({"metric": "vocab-sharded step of one rank, shards emulated on one GPU",
          "config": {"workload": "cfg4", "rows": rows, "vocab": vocab, "n_shards": n,
                     "shard_width": width, "temperature": cfg.temperature,
                     "top_k": cfg.top_k, "top_p": cfg.top_p},
          "steps": steps, "warmup": args.warmup,
          "partial_us": t_one, "partial_gbs": rows * width * 4 / (t_one * 1e-6) / 1e9,
          "partial_frac": rows * width * 4 / (t_one * 1e-6) / 1e9 / peak,
          "merge_us": t_merge, "record_bytes_per_row": rb,
          "rank_step_us_without_allgather": t_one + t_merge,
          "unsharded_us": t_unsharded,
          "strong_scaling_eff_without_allgather": t_unsharded / (n * (t_one + t_merge)),
          "bit_exact_vs_unsharded": bool(same)})


def lmhead_table(args) -> None:
    """Times the LM-head paths on one GPU (or tensor-parallel over the ranks):
    rsc_lmhead_sample (the GEMM with the sampler fused into its epilogue),
    rsc_lmhead_logits + rsc_sample, and the cuBLAS bf16 GEMM (torch.matmul) +
    rsc_sample, for a Qwen2.5-sized head (vocab 151936, dim 4096, bf16
    weights) at T 0.8, top-k 40, top-p 0.95. Seeded random weights and hidden
    states (no checkpoint). CUDA events over `steps` back-to-back calls after
    `warmup` calls. Prints one JSON line with a row per batch size."""
    import torch

    from rusticide_b200 import SamplingParams, engine

    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    vocab, dim = 151936, 4096
    params = SamplingParams(0.8, 40, 0.95)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / args.steps * 1000.0

    eng = engine(local)
    table = []
    if world > 1:
        from datetime import timedelta

        import torch.distributed as dist

        from rusticide_b200.sharding import VocabShardedSampler
        dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
        try:
            vs = VocabShardedSampler(eng, vocab)
            g = torch.Generator(device=dev).manual_seed(1 + rank)
            w = (torch.randn(vs.width, dim, device=dev, generator=g) * (3.0 / dim ** 0.5)).bfloat16()
            for rows in args.lmhead_rows:
                gh = torch.Generator(device=dev).manual_seed(7)  # the same hidden states everywhere
                h = torch.randn(rows, dim, device=dev, generator=gh).bfloat16()
                u = torch.rand(rows, device=dev, generator=gh)
                eng.ensure(rows, vocab)
                outs = eng._outputs(rows, True)
                t = torch.tensor([timed(lambda: vs.sample_lmhead(h, w, params, uniforms=u, out=outs))],
                                 device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                table.append({"rows": rows, "tensor_parallel_fused_us": float(t.item()),
                              "vocab_rows_per_rank": vs.width})
        finally:
            dist.destroy_process_group()
    else:
        g = torch.Generator(device=dev).manual_seed(1)
        w = (torch.randn(vocab, dim, device=dev, generator=g) * (3.0 / dim ** 0.5)).bfloat16()
        for rows in args.lmhead_rows:
            h = torch.randn(rows, dim, device=dev, generator=g).bfloat16()
            u = torch.rand(rows, device=dev, generator=g)
            eng.ensure(rows, vocab)
            outs = eng._outputs(rows, True)
            fused = timed(lambda: eng.lmhead_sample(h, w, params, uniforms=u, out=outs))
            flops = 2.0 * rows * dim * vocab
            row = {"rows": rows, "fused_us": fused, "fused_tflops": flops / fused / 1e6,
                   "weights_gbs": vocab * dim * 2 / fused / 1e3}
            if not args.fused_only:
                logits = eng.lmhead_logits(h, w)
                row["lmhead_logits_us"] = timed(lambda: eng.lmhead_logits(h, w))
                row["rsc_sample_us"] = timed(lambda: eng.sample(logits, params, uniforms=u, out=outs))
                row["cublas_bf16_us"] = timed(lambda: torch.matmul(h, w.T))
            table.append(row)
    if rank == 0:
        emit({"metric": "LM-head sampling us per call", "config": {"workload": "lmhead",
              "vocab": vocab, "dim": dim, "temperature": 0.8, "top_k": 40, "top_p": 0.95},
              "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "table": table})


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
    ap.add_argument("--sustained-seconds", type=float, default=1.0)
    ap.add_argument("--rows", type=int, default=0,
                    help="rows per GPU (default: the config's); for small profiling captures")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the parity, sustained and vocab-sharded legs (profiling captures)")
    ap.add_argument("--lmhead-rows", type=int, nargs="+", default=[1, 16, 64, 256, 1024])
    ap.add_argument("--emulate-shards", type=int, default=0,
                    help="--config cfg4 on one GPU: time one rank's partial pass and the merge "
                         "of N shards emulated on this GPU")
    ap.add_argument("--fused-only", action="store_true",
                    help="--config lmhead: time only rsc_lmhead_sample (profiling captures)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)

    if args.config == "lmhead":
        lmhead_table(args)
        return
    if args.emulate_shards > 0:
        if args.config != "cfg4" or world != 1 or args.impl != "ours":
            raise SystemExit("--emulate-shards runs --config cfg4 on one GPU (our arm)")
        emulated_shards(args)
        return

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
    peak, peak_kind = measured_peak()
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

    # Sustained: the same step for about --sustained-seconds (the number of
    # steps is fixed beforehand from the timed region's rate, so every rank
    # runs the same count), with the clocks sampled meanwhile.
    sus_steps = 0
    sus_ms = None
    sus_window = (0.0, 0.0)
    if not args.no_extras and args.sustained_seconds > 0 and args.steps > 0:
        per_step_s = max(t_ms / 1000.0 / args.steps, 1e-6)
        sus_steps = max(1, min(200000, int(args.sustained_seconds / per_step_s)))
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        sw0 = time.time()
        s0.record(stream)
        for _ in range(sus_steps):
            step()
        s1.record(stream)
        torch.cuda.synchronize(device)
        sus_window = (sw0, time.time())
        sus_ms = s0.elapsed_time(s1)
        barrier()

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
    clk = clocks.stop([("timed region", (wall0, wall1)),
                       (f"sustained region ({sus_steps} steps right after the timed region, "
                        f"which is shorter than the 50 ms sampling period)", sus_window)])
    call_ms = statistics.mean(a.elapsed_time(b) for a, b in per) if per else 0.0

    # End to end through the host-buffer entry point: H2D of the logits and
    # uniforms, sampling, D2H of ids, statuses and probabilities, every step.
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
    del x_host

    t_max = t_ms
    e2e_max = e2e_s
    sus_max = sus_ms
    if world > 1:
        tt = torch.tensor([t_ms, e2e_s, sus_ms or 0.0], dtype=torch.float64, device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_max, e2e_max = float(tt[0]), float(tt[1])
        sus_max = float(tt[2]) if sus_ms is not None else None

    # Correctness counters (rank 0, outside every timed region), then the
    # vocab-sharded leg (every rank), then the CPU baseline (rank 0, N = 1).
    parity = None
    if rank == 0 and not args.no_extras and not sharded:
        params_p = SamplingParams(0.0, cfg.top_k, cfg.top_p) if cfg.greedy else params
        parity = parity_counters(eng, cfg, params_p, device)
    barrier()
    vsh = None
    if not args.no_extras and not sharded:
        del x
        torch.cuda.empty_cache()
        vsh = vocab_sharded_leg(eng, world, rank, local, device, max(args.steps, 20),
                                args.warmup, peak)
    cpu = None
    if rank == 0 and world == 1:
        params_cpu = SamplingParams(0.0, cfg.top_k, cfg.top_p) if cfg.greedy else params
        xs, us = cpu_sample(cfg)
        cpu = cpu_baseline(xs, us, params_cpu, args.cpu_seconds, os.cpu_count() or 1, cfg.greedy)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return

    job_rows = rows if sharded else rows * world
    total_rows = job_rows * args.steps
    value = total_rows / (t_max / 1000.0)
    width = vs.width if sharded else vocab
    alg_bytes = rows * width * 4
    # The dominant kernel's average duration per launch over the timed region
    # (this rank's CUDA events on the launching stream). One sampling launch
    # per step; consecutive launches overlap by programmatic dependent launch,
    # so this is the steady-state cost.
    launches_per_step = launches / args.steps if args.steps else 0
    step_s = t_ms / 1000.0 / args.steps
    achieved = alg_bytes / step_s / 1e9
    single = alg_bytes / (call_ms / 1000.0) / 1e9 if call_ms else None
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
        "config": workload_config(cfg, rows, world, sharded),
        "hbm_gbs": achieved,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "launches_per_step": launches_per_step,
                     "single_call_gbs": single,
                     "single_call_us": call_ms * 1000.0,
                     "note": ("achieved = rows*vocab*4 B per step / CUDA-event time per step over "
                              "the timed region; single_call_* = one call bracketed by its own "
                              "events (no overlap with the next call); traffic = DRAM read+write "
                              "bytes per launch from the committed ncu summary in profiles/ "
                              "(captured on fewer rows and scaled by rows, as that file states)")},
        "e2e": {"value": job_rows * args.e2e_steps / e2e_max, "unit": "rows/s",
                "h2d_bytes_per_step": (rows * width * 4 if sharded else
                                       rows * vocab * 4 + (0 if cfg.greedy else rows * 4)),
                "d2h_bytes_per_step": rows * 12},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if sus_max is not None:
        sus_step_s = sus_max / 1000.0 / sus_steps
        line["sustained"] = {"steps": sus_steps, "seconds": sus_max / 1000.0,
                             "ms_per_step": sus_max / sus_steps,
                             "value": job_rows / sus_step_s, "unit": "rows/s",
                             "frac": alg_bytes / sus_step_s / 1e9 / peak}
    if parity is not None:
        line["parity"] = parity
    if vsh is not None:
        line["vocab_sharded"] = vsh
    if cpu is not None:
        line["cpu_baseline"] = cpu
    emit(line)


if __name__ == "__main__":
    main()
