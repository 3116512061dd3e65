"""Log-probability outputs of rsc_sample_ex (ABI 2): each row's log-sum-exp of
its scaled logits over the whole vocabulary, the chosen token's
log-probability and the survivors' ones, checked against a float64 CPU
log-sum-exp. The reference returns none of these (its softmax,
crates/rusticide-sampling/src/filters.rs:5-15, normalises over the survivors
only); they must also leave the sampling itself unchanged, bit for bit."""

import numpy as np
import pytest
import torch

from rusticide_b200 import SamplingParams, engine, synth

pytestmark = pytest.mark.gpu

# |got - want| <= TOL * max(1, |want|): the sums use the fast binary32 exp.
TOL = 1e-5


def scaled(x: np.ndarray, temperature: float) -> np.ndarray:
    """The reference's scaled logits (candidates.rs:25-37): NaN -> -inf, then
    x * (1/T) in binary32 for T > 0."""
    s = np.float32(1.0) / np.float32(temperature) if temperature > 0 else np.float32(1.0)
    v = np.where(np.isnan(x), np.float32(-np.inf), x).astype(np.float32) * s
    return v.astype(np.float32)


def lse64(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.float64)
    m = np.max(v, axis=1, keepdims=True)
    return (m[:, 0] + np.log(np.sum(np.exp(v - m), axis=1)))


def close(got, want) -> bool:
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return bool(np.all(np.abs(got - want) <= TOL * np.maximum(1.0, np.abs(want))))


@pytest.mark.parametrize("name,rows,params", [
    ("cfg2p", 24, SamplingParams(0.8, 40, 0.95)),      # streaming kernel, fused pass
    ("cfg2p", 8, SamplingParams(0.8, 200, 0.95)),      # k above the streaming filter: extra pass
    ("cfg3", 16, SamplingParams(1.0, 0, 0.95)),        # top-p only: large kernel
    ("cfg1_temp", 4, SamplingParams(0.7, 0, 1.0)),     # no filter: large kernel
    ("cfg0", 1, SamplingParams(0.8, 40, 0.95)),        # one row, whole
])
def test_logprobs_match_float64(name, rows, params):
    eng = engine(0)
    cfg = synth.CONFIGS[name]
    x = synth.make_config(cfg, rows=rows, base_seed=777)
    u = synth.uniforms(rows, seed=31)
    xd = torch.from_numpy(x).cuda()
    ud = torch.from_numpy(u).cuda()
    cap = 64
    base = eng.sample_ex(xd, params, uniforms=ud, survivor_cap=cap)
    out = eng.sample_ex(xd, params, uniforms=ud, survivor_cap=cap, logprobs=True)
    torch.cuda.synchronize()
    # The sampling is unchanged by the extra outputs.
    for a, b in zip(base, out[:6]):
        assert torch.equal(a.view(torch.int32) if a.dtype == torch.float32 else a,
                           b.view(torch.int32) if b.dtype == torch.float32 else b)
    ids, st, _, nsurv, surv, _, lse, tok, surv_lp = out
    v = scaled(x, params.temperature)
    want_lse = lse64(v)
    assert close(lse.cpu().numpy(), want_lse), name
    ids_h = ids.cpu().numpy().view(np.uint32)
    st_h = st.cpu().numpy() & 0xFF
    for r in range(rows):
        if st_h[r] == 0:
            assert close(tok.cpu().numpy()[r], v[r, ids_h[r]].astype(np.float64) - want_lse[r])
        n = min(int(nsurv[r]), cap)
        sid = surv[r, :n].cpu().numpy().view(np.uint32)
        assert close(surv_lp[r, :n].cpu().numpy(), v[r, sid].astype(np.float64) - want_lse[r])
