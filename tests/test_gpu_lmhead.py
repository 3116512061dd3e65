"""LM-head GEMM with the sampler fused into its epilogue (rsc_lmhead_*).

1. rsc_lmhead_logits against an f32 reference of the same product: bf16 x
   bf16 products are exact in f32, so the only difference is the order of the
   f32 sums, bounded by 2 * dim * 2^-24 * (|H| . |W|^T) per entry.
2. rsc_lmhead_sample against rsc_sample on the logits rsc_lmhead_logits
   returns: ids, statuses and probability bits identical (the fused epilogue
   sees the same f32 values), and those rows match the oracle
   (crates/rusticide-sampling/src/sampler.rs:44-54).
"""

import numpy as np
import pytest
import torch

from rusticide_b200 import SamplingParams, engine
from rusticide_b200.sampler import SamplingError

pytestmark = pytest.mark.gpu

# (rows, dim, vocab): partial row tiles, a dim that is not a multiple of 64,
# partial vocab tiles, and a Qwen-sized vocab shard. Up to 64 rows take the
# swapped-operand kernel (batch padded to 16, 32, 48 or 64), more rows the
# row-tile kernel.
SHAPES = [(1, 64, 300), (5, 256, 4096), (17, 136, 777), (64, 512, 18992), (65, 256, 3000),
          (130, 1000, 5000)]


def _inputs(rows, dim, vocab, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    h = torch.randn(rows, dim, device="cuda", generator=g).bfloat16()
    w = (torch.randn(vocab, dim, device="cuda", generator=g) * (3.0 / dim ** 0.5)).bfloat16()
    # A few boosted vocabulary rows give peaked rows, as an LM head does.
    hot = torch.randint(0, vocab, (8,), device="cuda", generator=g)
    w[hot] = (w[hot].float() * 4.0).bfloat16()
    return h, w


@pytest.fixture(scope="module")
def eng():
    return engine(0)


@pytest.mark.parametrize("rows,dim,vocab", SHAPES)
def test_lmhead_logits_match_f32_product(eng, rows, dim, vocab):
    h, w = _inputs(rows, dim, vocab, seed=rows * 131 + dim)
    got = eng.lmhead_logits(h, w)
    torch.cuda.synchronize()
    hf, wf = h.float(), w.float()
    want = hf @ wf.T
    bound = 2.0 * dim * 2.0 ** -24 * (hf.abs() @ wf.abs().T) + 1e-30
    err = (got - want).abs()
    assert torch.isfinite(got).all()
    assert (err <= bound).all(), f"max err {err.max().item()} vs bound {bound.max().item()}"


@pytest.mark.parametrize("rows,dim,vocab", SHAPES)
@pytest.mark.parametrize("temperature,top_k,top_p", [(0.8, 40, 0.95), (0.3, 40, 0.9),
                                                     (1.0, 1, 1.0), (1.5, 8, 1.0)])
def test_lmhead_sample_matches_sample_on_its_logits(eng, rows, dim, vocab, temperature, top_k,
                                                    top_p):
    h, w = _inputs(rows, dim, vocab, seed=rows * 17 + dim + vocab)
    params = SamplingParams(temperature, top_k, top_p)
    g = torch.Generator(device="cuda").manual_seed(5)
    u = torch.rand(rows, device="cuda", generator=g)
    ids_f, st_f, pr_f = eng.lmhead_sample(h, w, params, uniforms=u)
    logits = eng.lmhead_logits(h, w)
    ids_s, st_s, pr_s = eng.sample(logits, params, uniforms=u)
    torch.cuda.synchronize()
    assert torch.equal(st_f, st_s)
    assert torch.equal(ids_f, ids_s)
    assert torch.equal(pr_f.view(torch.int32), pr_s.view(torch.int32))
    assert (st_f & 0xFF).eq(0).all()

    from oracle import oracle as O
    x = logits.cpu().numpy()
    ref = O.sample_rows(x, O.params(temperature, top_k, top_p), u.cpu().numpy(), threads=4)
    assert np.array_equal(ids_f.cpu().numpy().astype(np.int64), ref["token"].astype(np.int64))


def test_lmhead_rejects_unsupported_params(eng):
    h, w = _inputs(2, 64, 300, seed=1)
    u = torch.rand(2, device="cuda")
    for params in (SamplingParams(0.8, 0, 0.95), SamplingParams(0.8, 100, 0.95),
                   SamplingParams(float("inf"), 40, 0.95)):
        with pytest.raises(Exception):
            eng.lmhead_sample(h, w, params, uniforms=u)
    with pytest.raises(SamplingError):
        eng.lmhead_logits(h.float(), w)


def test_lmhead_tied_row_reports_internal(eng):
    """A zero hidden state makes every logit of its row +0: each vocabulary
    part ties far beyond its record's capacity, so the row reports
    RSC_ROW_INTERNAL (to be resampled from rsc_lmhead_logits + rsc_sample),
    and the other rows of the batch are unaffected."""
    from rusticide_b200 import _lib
    h, w = _inputs(4, 256, 4096, seed=3)
    h[2] = 0
    params = SamplingParams(0.8, 40, 0.95)
    u = torch.rand(4, device="cuda")
    ids_f, st_f, pr_f = eng.lmhead_sample(h, w, params, uniforms=u)
    ids_s, st_s, pr_s = eng.sample(eng.lmhead_logits(h, w), params, uniforms=u)
    torch.cuda.synchronize()
    assert int(st_f[2]) & 0xFF == _lib.RSC_ROW_INTERNAL
    keep = torch.tensor([0, 1, 3], device="cuda")
    assert torch.equal(st_f[keep], st_s[keep])
    assert torch.equal(ids_f[keep], ids_s[keep])
    assert torch.equal(pr_f[keep].view(torch.int32), pr_s[keep].view(torch.int32))


@pytest.mark.parametrize("rows,dim,vocab,n_shards", [(1, 64, 300, 2), (5, 256, 4096, 2),
                                                     (64, 512, 18992, 3), (130, 256, 5000, 4)])
def test_lmhead_partial_shards_merge_to_the_fused_call(eng, rows, dim, vocab, n_shards):
    """A tensor-parallel LM head emulated on one GPU: each vocabulary shard of W
    through rsc_lmhead_partial, the records concatenated in shard order (what
    the all-gather produces) and merged by rsc_shard_merge, must give the
    tokens, statuses and probability bits of rsc_lmhead_sample on the whole W."""
    from rusticide_b200.sharding import vocab_shard
    h, w = _inputs(rows, dim, vocab, seed=rows * 3 + vocab)
    params = SamplingParams(0.8, 40, 0.95)
    g = torch.Generator(device="cuda").manual_seed(11)
    u = torch.rand(rows, device="cuda", generator=g)
    recs = []
    for r in range(n_shards):
        off, width = vocab_shard(vocab, n_shards, r)
        recs.append(eng.lmhead_partial(h, w[off:off + width], off, vocab, params).clone())
    gathered = torch.cat(recs)
    ids_m, st_m, pr_m = eng.shard_merge(gathered, n_shards, rows, vocab, params, uniforms=u)
    ids_f, st_f, pr_f = eng.lmhead_sample(h, w, params, uniforms=u)
    torch.cuda.synchronize()
    assert torch.equal(st_m, st_f)
    assert torch.equal(ids_m, ids_f)
    assert torch.equal(pr_m.view(torch.int32), pr_f.view(torch.int32))
    assert (st_m & 0xFF).eq(0).all()


@pytest.mark.parametrize("rows", [64, 256])
def test_lmhead_qwen_shape(eng, rows):
    """The Qwen2.5 LM head at full size, vocab 151936 x dim 4096 (the product
    crates/rusticide-transformer/src/decoder.rs:104-105 forms), through both
    kernels (up to 64 rows the swapped-operand one, above it the row-tile
    one): the logits are within the f32 bound of the product, the fused call
    equals rsc_sample on them bit for bit, and 16 rows match the oracle."""
    dim, vocab = 4096, 151936
    h, w = _inputs(rows, dim, vocab, seed=rows + 4096)
    params = SamplingParams(0.8, 40, 0.95)
    g = torch.Generator(device="cuda").manual_seed(rows)
    u = torch.rand(rows, device="cuda", generator=g)
    ids_f, st_f, pr_f = eng.lmhead_sample(h, w, params, uniforms=u)
    logits = eng.lmhead_logits(h, w)
    ids_s, st_s, pr_s = eng.sample(logits, params, uniforms=u)
    torch.cuda.synchronize()
    assert torch.equal(st_f, st_s)
    assert torch.equal(ids_f, ids_s)
    assert torch.equal(pr_f.view(torch.int32), pr_s.view(torch.int32))
    assert (st_f & 0xFF).eq(0).all()

    hf = h.float()
    for c0 in range(0, vocab, 32768):
        wf = w[c0:c0 + 32768].float()
        want = hf @ wf.T
        bound = 2.0 * dim * 2.0 ** -24 * (hf.abs() @ wf.abs().T) + 1e-30
        assert ((logits[:, c0:c0 + 32768] - want).abs() <= bound).all(), f"columns from {c0}"

    from oracle import oracle as O
    x = logits[:16].cpu().numpy()
    ref = O.sample_rows(x, O.params(0.8, 40, 0.95), u[:16].cpu().numpy(), threads=4)
    assert np.array_equal(ids_f[:16].cpu().numpy().astype(np.int64), ref["token"].astype(np.int64))
