"""Parity of the CUDA sampler (through the C ABI) with the CPU oracle.

Bar: statuses, token ids, survivor sets and probability bits identical to the
oracle on the same logits and uniforms. Every sum in the engine replays the
reference's sequential binary32 order, and its exp reproduces glibc's expf,
so no tolerance is needed; the north-star tolerances (probabilities 1e-5
relative, draws within 1e-6 of a CDF edge) are asserted as well, as the
looser contract.
"""

import math

import numpy as np
import pytest
import torch

from oracle import oracle as O
from rusticide_b200 import SamplingParams, engine, synth
from tests import kat

pytestmark = pytest.mark.gpu

PROB_RTOL = 1e-5   # north-star tolerance on probabilities
EDGE = 1e-6        # north-star tolerance on a draw's distance to a CDF edge


@pytest.fixture(scope="module")
def eng():
    if not torch.cuda.is_available():
        pytest.fail("gpu tests need CUDA")
    return engine(0)


def dev(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


# ---------------------------------------------------------------------------
# Reference known-answer tests on the device
# ---------------------------------------------------------------------------
class GpuBackend:
    def __init__(self, e):
        self.e = e

    def sample_logits(self, x, params, u):
        t, k, p = params
        x2 = dev(np.asarray(x, dtype=np.float32).reshape(1, -1))
        ids, st, _ = self.e.sample(x2, SamplingParams(t, k, p), uniforms=dev(np.array([u])))
        return int(st[0]) & 0xFF, int(ids[0])

    def greedy(self, x):
        x2 = dev(np.asarray(x, dtype=np.float32).reshape(1, -1))
        ids, st = self.e.greedy(x2)
        return int(st[0]) & 0xFF, int(ids[0])

    def with_temp(self, x, t, u):
        x2 = dev(np.asarray(x, dtype=np.float32).reshape(1, -1))
        ids, st, _ = self.e.sample_with_temp(x2, t, uniforms=dev(np.array([u])))
        return int(st[0]) & 0xFF, int(ids[0])

    def filter(self, x, params):
        t, k, p = params
        x2 = dev(np.asarray(x, dtype=np.float32).reshape(1, -1))
        n = max(1, x2.shape[1])
        _, _, _, ns, surv, _ = self.e.sample_ex(x2, SamplingParams(t, k, p),
                                             uniforms=dev(np.array([0.5])), survivor_cap=n)
        m = int(ns[0])
        return surv[0, :m].cpu().numpy(), None


def test_reference_kats_on_gpu(eng):
    assert kat.run_all(GpuBackend(eng)) >= 860


def test_greedy_kats_batched(eng):
    cases = kat.load()["greedy_logits"]
    for c in cases:
        x = kat.logits_of(c["logits"])
        if x.size == 0:
            continue
        ids, st = eng.greedy(dev(np.stack([x, x, x])))
        kat.check_result(c, int(st[1]) & 0xFF, int(ids[1]), c["src"])


# ---------------------------------------------------------------------------
# Differential sweep (the shape of candidates_tests.rs:172-201)
# ---------------------------------------------------------------------------
def reference_like_row(seed: int, vocab: int = 1000) -> np.ndarray:
    """The distribution of random_logits (candidates_tests.rs:135-152): 5% NaN,
    5% -inf, 10% duplicates of an earlier logit, otherwise k/100 - 10 for k
    in [0, 2000), and +inf at one position every 50 seeds. The reference draws
    it with fastrand; this uses numpy's PCG64."""
    rng = np.random.default_rng(seed ^ 0x5EED)
    out = np.empty(vocab, dtype=np.float32)
    for i in range(vocab):
        roll = rng.integers(0, 100)
        if roll < 5:
            out[i] = np.nan
        elif roll < 10:
            out[i] = -np.inf
        elif roll < 20 and i > 0:
            out[i] = out[rng.integers(0, i)]
        else:
            out[i] = np.float32(np.float32(rng.integers(0, 2000)) / np.float32(100.0)) - np.float32(10.0)
    if seed % 50 == 0:
        out[rng.integers(0, vocab)] = np.inf
    return out


def compare(eng, x: np.ndarray, params: SamplingParams, u: np.ndarray, tag: str,
            check_surv: bool = True, rows_subset=None) -> dict:
    """Runs the engine and the oracle on the same rows; asserts parity."""
    rows, vocab = x.shape
    cap = vocab if check_surv else 0
    ids, st, probs, ns, surv, survp = eng.sample_ex(dev(x), params, uniforms=dev(u), survivor_cap=cap)
    ids = ids.cpu().numpy().view(np.uint32)
    st = st.cpu().numpy()
    probs = probs.cpu().numpy()
    ns = ns.cpu().numpy()
    surv = surv.cpu().numpy()
    survp = survp.cpu().numpy()
    op = O.params(params.temperature, params.top_k, params.top_p)
    want = O.sample_rows(x, op, u, threads=8)
    stats = {"rows": rows, "edge": 0}
    for r in (range(rows) if rows_subset is None else rows_subset):
        w = want[r]
        code = int(st[r]) & 0xFF
        assert code == int(w["status"]), f"{tag} row {r}: status {code} != {w['status']}"
        if code != 0:
            continue
        assert ids[r] == w["token"], f"{tag} row {r}: token {ids[r]} != {w['token']} (u={u[r]})"
        wp, gp = np.float32(w["prob"]), np.float32(probs[r])
        if not (math.isnan(wp) and math.isnan(gp)):
            assert gp.view(np.uint32) == wp.view(np.uint32), f"{tag} row {r}: prob {gp!r} != {wp!r}"
            assert abs(gp - wp) <= PROB_RTOL * abs(wp)
        if int(st[r]) & 0x100:
            stats["edge"] += 1
        if check_surv:
            idx, vals = O.filter_(x[r], op)
            assert ns[r] == len(idx), f"{tag} row {r}: {ns[r]} survivors != {len(idx)}"
            assert np.array_equal(surv[r, :len(idx)].view(np.uint32), idx), f"{tag} row {r}: survivor ids"
            # The survivors' probabilities: the reference's softmax vector, bit
            # for bit (any NaN matches any NaN: x86 and CUDA differ in the sign
            # and payload of the NaNs they create).
            got_p, want_p = survp[r, :len(idx)], O.softmax(vals)
            nan = np.isnan(want_p)
            assert np.array_equal(np.isnan(got_p), nan), f"{tag} row {r}: survivor prob NaNs"
            assert np.array_equal(got_p[~nan].view(np.uint32), want_p[~nan].view(np.uint32)), \
                f"{tag} row {r}: survivor probs"
    return stats


TEMPS = [0.0, 0.7, 1.3]
TOPKS = [0, 1, 40, 1000, 5000]
TOPPS = [0.5, 0.95, 1.0]


def test_differential_sweep(eng):
    rows = np.stack([reference_like_row(s) for s in range(200)])
    u = synth.uniforms(200, seed=7)
    for t in TEMPS:
        for k in TOPKS:
            for p in TOPPS:
                compare(eng, rows, SamplingParams(t, k, p), u, f"T={t} k={k} p={p}")
    ids, st = eng.greedy(dev(rows))
    want = O.greedy_rows(rows)
    assert np.array_equal(st.cpu().numpy() & 0xFF, want["status"])
    ok = want["status"] == 0
    assert np.array_equal(ids.cpu().numpy().view(np.uint32)[ok], want["token"][ok])


def test_differential_sweep_large_path(eng):
    # vocab above the shared-memory survivor capacity with top-k off: every
    # row takes the large-survivor kernel (radix sort + exact replays).
    rows = np.stack([reference_like_row(s, 6000) for s in range(40)])
    u = synth.uniforms(40, seed=8)
    for t in TEMPS:
        for k in [0, 6000, 9000]:
            for p in TOPPS:
                compare(eng, rows, SamplingParams(t, k, p), u, f"large T={t} k={k} p={p}")


def test_overflow_rows_go_large(eng):
    # Thousands of logits tied at the k-th value overflow the streaming
    # kernel's list; those rows must come back exact from the large kernel.
    rng = np.random.default_rng(3)
    x = np.full((6, 20000), 1.0, dtype=np.float32)
    x[:, rng.integers(0, 20000, 30)] = 3.0
    x[1] = rng.integers(0, 4, 20000).astype(np.float32)  # 4 values, massive ties
    u = synth.uniforms(6, seed=9)
    compare(eng, x, SamplingParams(0.8, 40, 0.95), u, "ties")
    compare(eng, x, SamplingParams(1.0, 40, 1.0), u, "ties-no-topp")


@pytest.mark.parametrize("temperature", [float("inf"), 1e-45, -2.0, float("nan")])
def test_degenerate_temperatures(eng, temperature):
    rows = np.stack([reference_like_row(s, 700) for s in range(50)])
    rows[:, 5] = 0.0
    rows[:, 6] = -0.0
    u = synth.uniforms(50, seed=10)
    for k in [0, 3, 40]:
        for p in [0.5, 1.0]:
            compare(eng, rows, SamplingParams(temperature, k, p), u, f"T={temperature} k={k} p={p}")


def test_signed_zero_threshold(eng):
    # kth value +0.0 keeps -0.0 too (IEEE -0.0 < +0.0 is false).
    x = np.array([[1.0, 0.0, -0.0, -1.0, 0.0, 2.0, -0.0]], dtype=np.float32)
    for k in [2, 3, 4, 5]:
        compare(eng, x, SamplingParams(1.0, k, 1.0), np.array([0.4], np.float32), f"zeros k={k}")


# ---------------------------------------------------------------------------
# Benchmark configurations at reduced row counts (full vocabulary widths)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name,rows", [("cfg0", 1), ("cfg1_temp", 6), ("cfg2", 12), ("cfg2p", 12),
                                       ("cfg3", 24), ("cfg4", 6)])
def test_configs_match_oracle(eng, name, rows):
    cfg = synth.CONFIGS[name]
    x = synth.make_config(cfg, rows=rows, base_seed=4242)
    u = synth.uniforms(rows, seed=11)
    params = SamplingParams(cfg.temperature, cfg.top_k, cfg.top_p)
    compare(eng, x, params, u, name, check_surv=True)


@pytest.mark.parametrize("rows,vocab,top_k", [(1, 1_000_000, 40), (4, 400_000, 40), (2, 262_144, 100),
                                             (3, 800_000, 8), (1, 1_000_000, 8)])
def test_split_rows_many_parts(eng, rows, vocab, top_k):
    """Small batches of long rows: the balanced schedule spreads each row over
    several CTAs (parts of at least 16 chunks; 8, 6, 4, 12 and 15 parts for
    these shapes on 148 SMs), and the last part to arrive merges the parts'
    records before the row is finished."""
    x = synth.make_logits(rows, vocab, base_seed=vocab + rows)
    u = synth.uniforms(rows, seed=rows)
    compare(eng, x, SamplingParams(0.8, top_k, 0.95), u, f"{rows}x{vocab} k={top_k}")


@pytest.mark.parametrize("name,rows", [("cfg0_greedy", 1), ("cfg1_greedy", 16)])
def test_greedy_configs(eng, name, rows):
    cfg = synth.CONFIGS[name]
    x = synth.make_config(cfg, rows=rows, base_seed=77)
    ids, st = eng.greedy(dev(x))
    want = O.greedy_rows(x)
    assert np.array_equal(st.cpu().numpy(), want["status"])
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), want["token"])


def test_greedy_ties_and_strides(eng):
    # A strided view (row_stride > vocab) with ties: last maximum wins.
    base = np.zeros((9, 40003), dtype=np.float32)
    base[:, 7] = 5.0
    base[:, 39000] = 5.0
    base[3, :] = np.nan
    base[4, 123] = np.inf
    t = dev(base)[:, 1:40001]
    ids, st = eng.greedy(t)
    want = O.greedy_rows(base[:, 1:40001])
    assert np.array_equal(st.cpu().numpy(), want["status"])
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), want["token"])


def test_misaligned_rows_stream_path(eng):
    # Row starts that are not 16-byte aligned exercise the scalar head/tail.
    x = synth.make_logits(5, 30011, base_seed=5)
    t = dev(np.pad(x, ((0, 0), (1, 2))))[:, 1:30012]
    u = synth.uniforms(5, seed=12)
    ids, st, probs = eng.sample(t, SamplingParams(0.8, 40, 0.95), uniforms=dev(u))
    want = O.sample_rows(x, O.params(0.8, 40, 0.95), u)
    assert np.array_equal(st.cpu().numpy() & 0xFF, want["status"])
    assert np.array_equal(ids.cpu().numpy().view(np.uint32), want["token"])


# ---------------------------------------------------------------------------
# Full-size headline shape: exact on a sample of rows, properties on all rows
# ---------------------------------------------------------------------------
def test_headline_full_size(eng):
    cfg = synth.CONFIGS["cfg2p"]
    g = torch.Generator(device="cuda").manual_seed(2026)
    x = torch.randn(cfg.rows, cfg.vocab, device="cuda", generator=g) * 2.0
    spikes = torch.randint(0, cfg.vocab, (cfg.rows, 25), device="cuda", generator=g)
    x.scatter_add_(1, spikes, 5.0 + 7.0 * torch.rand(cfg.rows, 25, device="cuda", generator=g))
    u = torch.rand(cfg.rows, device="cuda", generator=g)
    params = SamplingParams(cfg.temperature, cfg.top_k, cfg.top_p)
    ids, st, probs, ns, _, _ = eng.sample_ex(x, params, uniforms=u)
    st_h = st.cpu().numpy()
    assert np.all(st_h & 0xFF == 0)
    # Property: the chosen token is among the row's top-40 scaled logits.
    top = torch.topk(x, 40, dim=1).values[:, -1]
    chosen = x.gather(1, ids.long().unsqueeze(1)).squeeze(1)
    assert bool(torch.all(chosen >= top))
    assert bool(torch.all(ns >= 1)) and bool(torch.all(ns <= 40))
    # Exactness on a sample of rows.
    sample = np.random.default_rng(1).choice(cfg.rows, 24, replace=False)
    xs = x[torch.from_numpy(sample).cuda()].cpu().numpy()
    us = u[torch.from_numpy(sample).cuda()].cpu().numpy()
    want = O.sample_rows(xs, O.params(0.8, 40, 0.95), us, threads=8)
    got_ids = ids.cpu().numpy().view(np.uint32)[sample]
    assert np.array_equal(got_ids, want["token"])
    got_p = probs.cpu().numpy()[sample]
    assert np.array_equal(got_p.view(np.uint32), want["prob"].view(np.uint32))


# ---------------------------------------------------------------------------
# exp, generator, tensor-level mirror
# ---------------------------------------------------------------------------
def test_device_exp_is_glibc_expf_exhaustive(eng):
    """Every binary32 x in [-104, 0]: the device exp equals glibc expf."""
    from rusticide_b200 import _lib
    lib = _lib.lib()
    lo = np.float32(-0.0).view(np.uint32)
    hi = np.float32(-104.0).view(np.uint32)
    chunk = 1 << 26
    bad = 0
    for start in range(int(lo), int(hi) + 1, chunk):
        stop = min(int(hi) + 1, start + chunk)
        bits = np.arange(start, stop, dtype=np.uint32)
        x = bits.view(np.float32)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        _lib.check(lib.rsc_expf(xd.data_ptr(), yd.data_ptr(), x.size, None), "rsc_expf")
        want = O.expf(x)
        got = yd.cpu().numpy()
        bad += int(np.count_nonzero(got.view(np.uint32) != want.view(np.uint32)))
    assert bad == 0


def test_device_generator_matches_restatement(eng):
    from rusticide_b200 import Sampler
    x = np.linspace(0, 3, 50, dtype=np.float32)
    s = Sampler(12345)
    us = O.rng_stream(12345, 40)
    for i in range(40):
        tok = s.sample_logits(torch.from_numpy(x), SamplingParams(1.0, 0, 1.0))
        want = O.sample_logits(x, O.params(1.0, 0, 1.0), float(us[i]))
        assert tok == want.token
    # Greedy draws consume nothing; the next draw still follows the stream.
    s.sample_logits(torch.from_numpy(x), SamplingParams(0.0, 0, 1.0))
    s.greedy_logits(torch.from_numpy(x))
    us2 = O.rng_stream(12345, 41)
    tok = s.sample_logits(torch.from_numpy(x), SamplingParams(1.0, 0, 1.0))
    assert tok == O.sample_logits(x, O.params(1.0, 0, 1.0), float(us2[40])).token


def test_tensor_entry_points(eng):
    from rusticide_b200 import InvalidShape, NoValidTokens, Sampler, TensorError
    s = Sampler(42)
    assert s.sample_greedy(torch.tensor([[1.0, 2.0, 3.0, 4.0, 5.0]])) == 4  # logits.rs:46-52
    with pytest.raises(InvalidShape):
        s.sample(torch.zeros(2, 3, 4), SamplingParams())
    with pytest.raises(InvalidShape):
        s.sample(torch.zeros(2, 3), SamplingParams())
    with pytest.raises(TensorError):
        s.sample(torch.zeros(3, dtype=torch.float16), SamplingParams())
    with pytest.raises(NoValidTokens):
        s.sample(torch.zeros(0), SamplingParams())
    with pytest.raises(NoValidTokens):
        s.sample_greedy(torch.zeros(0))
    with pytest.raises(NoValidTokens):
        s.sample_with_temp(torch.zeros(0), 1.0)
    assert s.sample_with_temp(torch.tensor([-5.0, 100.0, -5.0]), 0.0) == 1
    row = torch.tensor([1.0, 1.0, 1.0, 1.0], device="cuda")
    s.penalize(row, [0, 2], 2.0)
    assert row.cpu().tolist() == [0.5, 1.0, 0.5, 1.0]


def test_penalize_matches_oracle(eng):
    x = synth.make_logits(3, 1000, base_seed=1)
    toks = np.array([5, 7, 5, 999, 1000, 4294967295], dtype=np.uint32)
    t = dev(x)
    eng.penalize(t, torch.from_numpy(toks.view(np.int32)), 1.3)
    for r in range(3):
        want = O.apply_repetition_penalty(x[r], toks, 1.3)
        assert np.array_equal(t[r].cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_pick_host_matches_device(eng):
    cfg = synth.CONFIGS["cfg0"]
    x = synth.make_config(cfg, rows=4, base_seed=3)
    u = synth.uniforms(4, seed=4)
    ids, st, probs = eng.pick_host(x, SamplingParams(0.8, 40, 0.95), u)
    want = O.sample_rows(x, O.params(0.8, 40, 0.95), u)
    assert np.array_equal(ids, want["token"])
    ids0, st0, _ = eng.pick_host(x, SamplingParams(0.0, 40, 0.95), None)
    assert np.array_equal(ids0, O.greedy_rows(x)["token"])


# ---------------------------------------------------------------------------
# Vocab-sharded merge, emulated on one GPU (each shard a column slice)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("n_shards,top_k", [(2, None), (4, None), (8, None), (10, 40), (16, 40),
                                             (8, 100), (4, 128)])
def test_vocab_sharded_matches_unsharded(eng, n_shards, top_k):
    """Shard records merged into the unsharded result. Up to n_shards * (k + 24)
    = 512 entries per row one warp merges them; beyond (10 and 16 shards at
    k 40, 8 at k 100, 4 at k 128) one block per row does. At k 100 and 128
    some shard rows overflow the streaming list and are rescued into their
    records by the partial pass's epilogue. Row 5 holds up to 40 values tied
    at its maximum in every shard (480 in all at most, within one finisher's
    list): from 4 shards on, more survive the keep test than a merging
    warp's lean workspace holds (128), and the row is merged again with the
    full one."""
    cfg = synth.CONFIGS["cfg4"]
    rows = 16
    x = synth.make_config(cfg, rows=rows, base_seed=606)
    x[3, 100:140] = 9.0   # ties across a shard boundary
    V = cfg.vocab
    bounds = [V * s // n_shards for s in range(n_shards + 1)]
    ties = min(40, 480 // n_shards)
    for s in range(n_shards):
        x[5, bounds[s] + 10:bounds[s] + 10 + ties] = 40.0  # ties at the row's maximum
    u = synth.uniforms(rows, seed=13)
    params = SamplingParams(cfg.temperature, top_k or cfg.top_k, cfg.top_p)
    xd = dev(x)
    recs = []
    for s in range(n_shards):
        shard = xd[:, bounds[s]:bounds[s + 1]]
        recs.append(eng.shard_partial(shard, bounds[s], V, params))
    gathered = torch.cat(recs)
    ids, st, probs = eng.shard_merge(gathered, n_shards, rows, V, params, uniforms=dev(u))
    ids0, st0, probs0 = eng.sample(xd, params, uniforms=dev(u))
    assert torch.equal(st, st0)
    assert torch.equal(ids, ids0)
    assert torch.equal(probs.view(torch.int32), probs0.view(torch.int32))


@pytest.mark.parametrize("top_k", [100, 128])
def test_large_k_rows_rescued_exactly(eng, top_k):
    """k near the streaming limit: the first chunks' bound can admit more
    candidates than the list holds. Such rows are finished in the CTA's
    epilogue by a histogram pass and a gather pass (the large-row code only
    when ties overflow the list too); every row must still match the oracle."""
    rows, vocab = 48, 151936
    x = synth.make_logits(rows, vocab, base_seed=4321)
    u = synth.uniforms(rows, seed=17)
    compare(eng, x, SamplingParams(0.8, top_k, 0.95), u, f"k{top_k}", check_surv=False)


@pytest.mark.parametrize("top_k,vocab,check_surv", [(200, 151936, False), (488, 151936, False),
                                                    (300, 32000, True)])
def test_topk_above_streaming_limit(eng, top_k, vocab, check_surv):
    """128 < k <= 488: rows are not streamed but finished by the two-pass
    top-k (histogram, gather, exact finisher) in the streaming kernel's
    epilogue; ids, probabilities and survivor sets must match the oracle."""
    rows = 24
    x = synth.make_logits(rows, vocab, base_seed=top_k)
    u = synth.uniforms(rows, seed=top_k + 1)
    compare(eng, x, SamplingParams(0.8, top_k, 0.95), u, f"k{top_k}", check_surv=check_surv)
