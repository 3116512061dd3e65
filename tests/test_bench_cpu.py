"""bench.py's output contract, checked on the CPU through its reference arm:
exactly one JSON line on stdout with the metric, the timing fields and the
reference arm's cpu_baseline and e2e objects. Everything else the run prints
(argparse, native libraries such as NCCL) belongs on stderr."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_json_line(oracle_lib):
    r = subprocess.run(
        [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", "cfg0",
         "--steps", "3", "--warmup", "3", "--ref-seconds", "5"],
        capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.splitlines()
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "config", "impl", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["steps"] == 3 and d["warmup"] == 3
    assert d["config"]["workload"] == "cfg0"
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] in ("port", "reference")


def test_headline_profile_gives_the_roofline_traffic():
    """roofline.traffic on the headline comes from the committed ncu summary's
    dram_bytes_per_launch line; a launch reads each logit at least once."""
    sys.path.insert(0, str(ROOT))
    import bench
    traffic = bench.committed_traffic("cfg2p")
    assert traffic is not None
    assert traffic >= 1024 * 151936 * 4


def test_cpu_baseline_reports_all_cores_and_one_core(oracle_lib):
    """The GPU arm's cpu_baseline (the oracle on the host cores) also carries a
    single-core figure; both are positive rates over bounded samples."""
    sys.path.insert(0, str(ROOT))
    import bench
    from rusticide_b200 import SamplingParams, synth
    x = synth.make_logits(16, 32000, base_seed=3)
    u = synth.uniforms(16, seed=4)
    out = bench.cpu_baseline(x, u, SamplingParams(0.8, 40, 0.95), 0.4, 4)
    assert out["value"] > 0 and out["single_core_value"] > 0
    assert out["cores"] == 4 and out["kind"] == "port" and out["unit"] == "rows/s"
    g = bench.cpu_baseline(x, u, SamplingParams(0.0, 40, 0.95), 0.2, 2, greedy=True)
    assert g["single_core_value"] > 0
