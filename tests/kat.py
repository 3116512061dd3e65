"""Runner of the reference's known-answer cases (tests/golden/reference_kats.json)
against a backend: the CPU oracle, or the CUDA engine through the C ABI.

A backend provides:
  sample_logits(logits, (T, k, p), u) -> (status, token)
  greedy(logits) -> (status, token)
  with_temp(logits, T, u) -> (status, token)
  filter(logits, (T, k, p)) -> (tokens, values) or None when not observable
"""

from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

KAT_PATH = Path(__file__).resolve().parent / "golden" / "reference_kats.json"
NO_VALID = "NoValidTokens"
OK = 0
NO_VALID_CODE = 1


def load() -> dict:
    return json.loads(KAT_PATH.read_text())


def f(v) -> float:
    if isinstance(v, str):
        return {"nan": math.nan, "inf": math.inf, "-inf": -math.inf}[v]
    return float(v)


def logits_of(spec) -> np.ndarray:
    if isinstance(spec, str):
        if spec.startswith("range:"):
            return np.arange(int(spec.split(":")[1]), dtype=np.float32)
        if spec.startswith("zeros:"):
            n, tail = spec.split(":")[1].split("+")
            a = np.zeros(int(n), dtype=np.float32)
            if tail == "nan":
                a = np.append(a, np.float32(np.nan))
            return a.astype(np.float32)
        raise ValueError(spec)
    return np.array([f(v) for v in spec], dtype=np.float32)


def draw_uniforms(case: dict, count: int) -> np.ndarray:
    if "uniforms" in case:
        return np.array(case["uniforms"], dtype=np.float32)
    rng = np.random.default_rng(20261201)
    u = rng.random(count, dtype=np.float32)
    lo = case.get("uniform_min")
    if lo is not None:
        u = np.maximum(u, np.float32(lo))
    # Always include the ends of [0, 1).
    return np.concatenate([u, np.array([0.0, 0.5, 0.99999994], dtype=np.float32)
                           if lo is None else np.array([0.5, 0.99999994], dtype=np.float32)])


def check_result(case: dict, status: int, token: int, what: str) -> None:
    if case.get("expect") == NO_VALID:
        assert status == NO_VALID_CODE, f"{what}: expected NoValidTokens, got status {status} token {token}"
        return
    assert status == OK, f"{what}: status {status}"
    if "expect_in" in case:
        assert token in case["expect_in"], f"{what}: token {token} not in {case['expect_in']}"
    else:
        assert token == case["expect"], f"{what}: token {token} != {case['expect']}"


def run_all(backend, include_filter: bool = True) -> int:
    """Runs every case; returns the number of checks made."""
    kats = load()
    n = 0
    for case in kats["sample_logits"]:
        x = logits_of(case["logits"])
        params = tuple(case["params"])
        draws = case.get("draws", 1)
        us = draw_uniforms(case, draws)
        for u in us:
            st, tok = backend.sample_logits(x, params, float(u))
            check_result(case, st, tok, f"sample_logits {case['src']} u={u}")
            n += 1
    sweep = kats["sample_logits_no_valid_sweep"]
    for inp in sweep["inputs"]:
        x = np.array([f(v) for v in inp], dtype=np.float32)
        for t in sweep["temperatures"]:
            for k in sweep["top_ks"]:
                for p in sweep["top_ps"]:
                    st, tok = backend.sample_logits(x, (t, k, p), 0.5)
                    assert st == NO_VALID_CODE, f"no-valid sweep {inp} T={t} k={k} p={p}: {st} {tok}"
                    n += 1
    for case in kats["greedy_logits"]:
        st, tok = backend.greedy(logits_of(case["logits"]))
        check_result(case, st, tok, f"greedy {case['src']}")
        n += 1
    for case in kats["sample_with_temp"]:
        x = logits_of(case["logits"])
        us = draw_uniforms(case, case.get("draws", 1))
        for u in us:
            st, tok = backend.with_temp(x, case["temperature"], float(u))
            check_result(case, st, tok, f"with_temp {case['src']} u={u}")
            n += 1
    for case in kats["same_draws"]:
        x = logits_of(case["logits"])
        for u in draw_uniforms(case, case["draws"]):
            a = backend.sample_logits(x, tuple(case["params_a"]), float(u))
            b = backend.sample_logits(x, tuple(case["params_b"]), float(u))
            assert a == b, f"same draws {case['src']} u={u}: {a} != {b}"
            n += 1
    if include_filter:
        for case in kats["filter"]:
            got = backend.filter(logits_of(case["logits"]), tuple(case["params"]))
            if got is None:
                continue
            toks, vals = got
            assert list(map(int, toks)) == case["tokens"], f"filter tokens {case['src']}: {toks}"
            if vals is not None:
                assert [float(v) for v in vals] == [float(v) for v in case["values"]], \
                    f"filter values {case['src']}: {vals}"
            n += 1
    prop = kats["mixed_nan_property"]
    state = prop["lcg_state"]
    T, k, p = prop["params"]
    for r in range(prop["rows"]):
        row = []
        for _ in range(prop["vocab"]):
            state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
            row.append(math.nan if (state >> 28) < 5 else float(np.float32(state >> 16) / np.float32(1000.0)))
        x = np.array(row, dtype=np.float32)
        u = float(np.float32((r * 0.61803398875) % 1.0))
        st, tok = backend.sample_logits(x, (T, k, p), u)
        assert st == OK and not math.isnan(row[tok]), f"mixed NaN row {r}: {st} {tok}"
        n += 1
    return n
