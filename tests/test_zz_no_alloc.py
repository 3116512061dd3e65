"""rsc_sample_noalloc: the allocation-free entry point for callers that cannot let
the library call cudaMalloc (a server that has reserved HBM for its KV cache,
a runtime with its own memory pool, a plugin with no place to free a handle).

It must give the same results as rsc_sample, call after call, although its
sorting scratch is one fixed device array shared by every call. This file is
collected last so that a failure here cannot hide the other tests' results.
"""

import ctypes

import numpy as np
import pytest
import torch

from rusticide_b200 import SamplingParams, _lib, engine, synth


def noalloc(x: torch.Tensor, params: SamplingParams, u, states=None):
    lib = _lib.lib()
    rows, vocab = x.shape
    ids = torch.empty(rows, dtype=torch.int32, device=x.device)
    st = torch.empty(rows, dtype=torch.int32, device=x.device)
    probs = torch.empty(rows, dtype=torch.float32, device=x.device)
    c = params.to_c()
    _lib.check(lib.rsc_sample_noalloc(x.data_ptr(), rows, vocab, x.stride(0), ctypes.byref(c),
                                      None if u is None else u.data_ptr(),
                                      None if states is None else states.data_ptr(),
                                      ids.data_ptr(), st.data_ptr(), probs.data_ptr(),
                                      torch.cuda.current_stream(x.device).cuda_stream),
               "rsc_sample_noalloc")
    return ids, st, probs


def test_rejects_vocab_above_the_scratch_limit():
    lib = _lib.lib()
    c = SamplingParams(1.0, 0, 0.95).to_c()
    out = ctypes.c_int32()
    rc = lib.rsc_sample_noalloc(ctypes.c_void_p(16), 1, _lib.RSC_NOALLOC_MAX_VOCAB + 1,
                                _lib.RSC_NOALLOC_MAX_VOCAB + 1, ctypes.byref(c), ctypes.c_void_p(16),
                                None, ctypes.byref(out), ctypes.byref(out), None, None)
    assert rc == _lib.RSC_ERR_CAPACITY


def test_rejects_an_empty_vocabulary():
    # Checked before any CUDA call, so it runs without a GPU.
    lib = _lib.lib()
    c = SamplingParams(1.0, 0, 0.95).to_c()
    out = ctypes.c_int32()
    rc = lib.rsc_sample_noalloc(ctypes.c_void_p(16), 3, 0, 0, ctypes.byref(c), ctypes.c_void_p(16),
                                None, ctypes.byref(out), ctypes.byref(out), None, None)
    assert rc == _lib.RSC_ERR_INVALID_SHAPE


def _slots(vocab: int, sms: int) -> int:
    """Rows one no-alloc launch samples at once (the kernel loops over the rest)."""
    return min(_lib.RSC_NOALLOC_SCRATCH_BYTES // (16 * vocab), 2 * sms)


@pytest.mark.gpu
def test_noalloc_matches_rsc_sample_on_two_calls_in_a_row():
    if not torch.cuda.is_available():
        pytest.fail("needs CUDA")
    eng = engine(0)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    flat = synth.CONFIGS["cfg3"]
    peaked = synth.CONFIGS["cfg2"]
    batches = [
        # top-p only over flat rows: the whole-row sort path
        (synth.make_config(flat, rows=40, base_seed=31), SamplingParams(1.0, 0, 0.95), "u"),
        # top-k 40 / top-p 0.95 on 64 rows of 128256: more rows than the
        # scratch holds at once (32), so each block reuses its slot
        (synth.make_config(peaked, rows=64, base_seed=32), SamplingParams(0.8, 40, 0.95), "u"),
        # no filter at all: the filter-free branch, as rsc_sample takes it
        (synth.make_config(peaked, rows=8, base_seed=33), SamplingParams(1.0, 0, 1.0), "u"),
        # argmax branch (T = 0): no uniform is read
        (synth.make_config(peaked, rows=6, base_seed=34), SamplingParams(0.0, 40, 0.95), None),
        # per-row generator states instead of uniforms
        (synth.make_config(flat, rows=12, base_seed=35), SamplingParams(0.7, 100, 0.9), "states"),
    ]
    assert _slots(peaked.vocab, sms) < 64
    for call, (x_host, params, draw) in enumerate(batches):
        x = torch.from_numpy(x_host).cuda()
        u = None
        st_a = st_b = None
        if draw == "u":
            u = torch.from_numpy(synth.uniforms(x.shape[0], seed=40 + call)).cuda()
        elif draw == "states":
            seeds = torch.arange(1000, 1000 + x.shape[0], dtype=torch.int64, device="cuda")
            st_a = eng.rng_seed(seeds)
            st_b = st_a.clone()
        want_ids, want_st, want_p = eng.sample(x, params, uniforms=u, rng_states=st_a)
        ids, st, probs = noalloc(x, params, u, st_b)
        torch.cuda.synchronize()
        assert torch.equal(st & 0xFF, want_st & 0xFF), f"call {call}: statuses"
        assert torch.equal(ids, want_ids), f"call {call}: token ids"
        # Probabilities: identical bits (the tests' bar), within 1e-5 relative a fortiori.
        assert torch.equal(probs.view(torch.int32), want_p.view(torch.int32)), f"call {call}: probs"
        if st_a is not None:
            assert torch.equal(st_a, st_b), f"call {call}: generator states"
