"""Seeded synthetic logits for the benchmark configurations and tests.

The reference publishes no sampling dataset; these rows stand in for LM-head
outputs with the shapes and value distributions of the benchmark configs:

  peaked: 2.0 * N(0,1) per logit, plus `spikes` distinct indices boosted by
          U(5, 12) (a peaked LM distribution);
  flat:   0.5 * N(0,1), no spikes (a nucleus covering most of the vocabulary).

Row r draws from numpy's PCG64 seeded with base_seed + r: Box-Muller-free
standard normals in float64, scaled and rounded once to float32; spike indices
are drawn without replacement from the same stream, then their U(5, 12)
boosts are added in float64 before rounding.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np


@dataclass(frozen=True)
class Config:
    name: str
    rows: int
    vocab: int
    temperature: float
    top_k: int
    top_p: float
    dist: str            # "peaked" or "flat"
    spikes: tuple        # (lo, hi) inclusive spike count per row; (0, 0) for none
    greedy: bool = False


# BASELINE.json "configs" (index = config number), plus the metric's 2' shape.
CONFIGS = {
    "cfg0": Config("cfg0", 1, 32000, 0.8, 40, 0.95, "peaked", (20, 20)),
    "cfg0_greedy": Config("cfg0_greedy", 1, 32000, 0.0, 40, 0.95, "peaked", (20, 20), greedy=True),
    "cfg1_greedy": Config("cfg1_greedy", 256, 151936, 0.0, 0, 1.0, "peaked", (20, 20), greedy=True),
    "cfg1_temp": Config("cfg1_temp", 256, 151936, 0.7, 0, 1.0, "peaked", (20, 20)),
    "cfg2": Config("cfg2", 1024, 128256, 0.8, 40, 0.95, "peaked", (1, 50)),
    "cfg2p": Config("cfg2p", 1024, 151936, 0.8, 40, 0.95, "peaked", (1, 50)),
    "cfg3": Config("cfg3", 4096, 32000, 1.0, 0, 0.95, "flat", (0, 0)),
    "cfg4": Config("cfg4", 8192, 151936, 0.8, 40, 0.95, "peaked", (20, 20)),
}


def _distinct(rng: np.random.Generator, n: int, k: int) -> np.ndarray:
    """k distinct indices in [0, n), drawn in order with rejection."""
    out: list[int] = []
    seen: set[int] = set()
    while len(out) < k:
        i = int(rng.integers(0, n))
        if i not in seen:
            seen.add(i)
            out.append(i)
    return np.array(out, dtype=np.int64)


def make_row(vocab: int, seed: int, dist: str = "peaked", spikes=(20, 20)) -> np.ndarray:
    rng = np.random.default_rng(seed)
    scale = 2.0 if dist == "peaked" else 0.5
    x = rng.standard_normal(vocab) * scale
    lo, hi = spikes
    if hi > 0 and vocab > 0:
        k = lo if lo == hi else int(rng.integers(lo, hi + 1))
        k = min(k, vocab)
        idx = _distinct(rng, vocab, k)
        x[idx] += rng.uniform(5.0, 12.0, size=k)
    return x.astype(np.float32)


def make_logits(rows: int, vocab: int, base_seed: int = 1234, dist: str = "peaked",
                spikes=(20, 20), out: Optional[np.ndarray] = None) -> np.ndarray:
    a = out if out is not None else np.empty((rows, vocab), dtype=np.float32)
    for r in range(rows):
        a[r] = make_row(vocab, base_seed + r, dist, spikes)
    return a


def make_config(cfg: Config, rows: Optional[int] = None, vocab: Optional[int] = None,
                base_seed: int = 1234) -> np.ndarray:
    return make_logits(rows if rows is not None else cfg.rows,
                       vocab if vocab is not None else cfg.vocab, base_seed, cfg.dist, cfg.spikes)


def uniforms(rows: int, seed: int = 99) -> np.ndarray:
    """Per-row draws in [0, 1) for tests and the benchmark (float32)."""
    rng = np.random.default_rng(seed)
    return rng.random(rows, dtype=np.float32)
