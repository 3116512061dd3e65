"""One parameter set per row (rsc_sample_rows).

Row r of a call must equal Sampler::sample_logits(row r, params[r])
(crates/rusticide-sampling/src/sampler.rs:44-54): the oracle on that row with
that set, and rsc_sample on the rows that share the set, with identical ids,
statuses, probability bits and generator states. The mix covers rows the
streaming filter serves and rows it leaves to the whole-row path (top-k off,
k above the streaming limit, T = inf) in the same launch.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from rusticide_b200 import SamplingParams, engine, synth

pytestmark = pytest.mark.gpu

MIX = [
    (0.8, 40, 0.95), (0.3, 40, 0.9), (0.0, 40, 0.9), (1.0, 1, 1.0), (1.5, 8, 1.0),
    (0.9, 128, 0.8),
    (0.7, 0, 1.0),             # temperature only: whole row
    (1.0, 0, 0.9),             # top-p only: whole row
    (0.0, 0, 1.0),             # argmax over the whole row
    (1.2, 200, 0.95),          # k above the streaming filter's limit
    (float("inf"), 40, 0.95),  # scale 0
]


@pytest.fixture(scope="module")
def eng():
    return engine(0)


def dev(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _choice(rows: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, len(MIX), rows)


def _groups(choice: np.ndarray):
    for m in np.unique(choice):
        yield int(m), np.nonzero(choice == m)[0]


@pytest.mark.parametrize("rows,vocab", [(7, 4096), (64, 151936), (300, 32000), (1000, 128256)])
def test_rows_match_oracle_and_per_set_calls(eng, rows, vocab):
    x = synth.make_logits(rows, vocab, base_seed=rows * 7 + vocab)
    u = synth.uniforms(rows, seed=rows)
    choice = _choice(rows, seed=vocab)
    ps = [SamplingParams(*MIX[m]) for m in choice]
    ids, st, pr = eng.sample_rows(dev(x), ps, uniforms=dev(u))
    torch.cuda.synchronize()
    ids = ids.cpu().numpy().view(np.uint32)
    st = st.cpu().numpy()
    pr = pr.cpu().numpy()
    for m, idx in _groups(choice):
        t, k, p = MIX[m]
        want = O.sample_rows(x[idx], O.params(t, k, p), u[idx], threads=8)
        gi, gs, gp = eng.sample(dev(x[idx]), SamplingParams(t, k, p), uniforms=dev(u[idx]))
        gi = gi.cpu().numpy().view(np.uint32)
        gs = gs.cpu().numpy()
        gp = gp.cpu().numpy()
        for j, r in enumerate(idx):
            tag = f"row {r} params {MIX[m]}"
            assert (st[r] & 0x1FF) == (gs[j] & 0x1FF), tag
            assert int(st[r]) & 0xFF == int(want[j]["status"]), tag
            if int(st[r]) & 0xFF:
                continue
            assert ids[r] == want[j]["token"] == gi[j], tag
            assert pr[r].view(np.uint32) == gp[j].view(np.uint32), tag
            wp = np.float32(want[j]["prob"])
            assert pr[r].view(np.uint32) == wp.view(np.uint32), tag


def test_one_set_for_every_row_equals_rsc_sample(eng):
    rows, vocab = 256, 151936
    x = dev(synth.make_logits(rows, vocab, base_seed=5))
    u = dev(synth.uniforms(rows, seed=6))
    params = SamplingParams(0.8, 40, 0.95)
    a = eng.sample_rows(x, [params] * rows, uniforms=u)
    b = eng.sample(x, params, uniforms=u)
    torch.cuda.synchronize()
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    assert torch.equal(a[2].view(torch.int32), b[2].view(torch.int32))


def test_rows_advance_generators_as_per_set_calls(eng):
    rows, vocab = 96, 32000
    x = synth.make_logits(rows, vocab, base_seed=11)
    choice = _choice(rows, seed=12)
    ps = [SamplingParams(*MIX[m]) for m in choice]
    seeds = torch.arange(1000, 1000 + rows, dtype=torch.int64, device="cuda")
    st_rows = eng.rng_seed(seeds)
    st_sets = st_rows.clone()
    for step in range(2):  # two calls: states carried from the first
        ids, st, pr = eng.sample_rows(dev(x), ps, rng_states=st_rows)
        for m, idx in _groups(choice):
            ti = torch.from_numpy(idx).cuda()
            sub = st_sets[ti].clone()
            gi, gs, gp = eng.sample(dev(x[idx]), SamplingParams(*MIX[m]), rng_states=sub)
            st_sets[ti] = sub
            assert torch.equal(ids[ti], gi), f"step {step} params {MIX[m]}"
            assert torch.equal(st[ti] & 0xFF, gs & 0xFF)
        torch.cuda.synchronize()
        assert torch.equal(st_rows, st_sets), f"step {step}: generator states"


def test_rows_reject_bad_arguments(eng):
    x = dev(synth.make_logits(4, 1000, base_seed=1))
    from rusticide_b200.sampler import SamplingError
    with pytest.raises(SamplingError):
        eng.sample_rows(x, [SamplingParams()] * 3)  # one set short
    with pytest.raises(Exception):
        eng.sample_rows(x, [SamplingParams()] * 4)  # draws need uniforms or states
    ids, st, _ = eng.sample_rows(x, [SamplingParams(0.0, 40, 0.9)] * 4)  # argmax rows need none
    torch.cuda.synchronize()
    assert (st & 0xFF).eq(0).all()


def test_rows_beyond_one_launch():
    """More rows than one streaming launch takes (148 SMs x 3 CTAs x 48 rows =
    21312 on a B200): the call is split into launches, and each launch must
    read the parameter sets of its own rows."""
    from rusticide_b200.sampler import Engine
    rows, vocab = 21412, 700
    eng = Engine(0, rows, vocab)  # its own handle: small staging buffers
    x = synth.make_logits(rows, vocab, base_seed=21)
    u = synth.uniforms(rows, seed=22)
    choice = _choice(rows, seed=23)
    ps = [SamplingParams(*MIX[m]) for m in choice]
    ids, st, pr = eng.sample_rows(dev(x), ps, uniforms=dev(u))
    torch.cuda.synchronize()
    for m, idx in _groups(choice):
        ti = torch.from_numpy(idx).cuda()
        gi, gs, gp = eng.sample(dev(x[idx]), SamplingParams(*MIX[m]), uniforms=dev(u[idx]))
        assert torch.equal(ids[ti], gi), f"params {MIX[m]}"
        assert torch.equal(st[ti] & 0x1FF, gs & 0x1FF)
        assert torch.equal(pr[ti].view(torch.int32), gp.view(torch.int32))
    eng.close()
