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


def noalloc(x: torch.Tensor, params: SamplingParams, u: torch.Tensor):
    lib = _lib.lib()
    rows, vocab = x.shape
    ids = torch.empty(rows, dtype=torch.int32, device=x.device)
    st = torch.empty(rows, dtype=torch.int32, device=x.device)
    probs = torch.empty(rows, dtype=torch.float32, device=x.device)
    c = params.to_c()
    _lib.check(lib.rsc_sample_noalloc(x.data_ptr(), rows, vocab, x.stride(0), ctypes.byref(c),
                                      u.data_ptr(), None, ids.data_ptr(), st.data_ptr(),
                                      probs.data_ptr(),
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


@pytest.mark.gpu
def test_noalloc_matches_rsc_sample_on_two_calls_in_a_row():
    if not torch.cuda.is_available():
        pytest.fail("needs CUDA")
    eng = engine(0)
    flat = synth.CONFIGS["cfg3"]
    peaked = synth.CONFIGS["cfg2"]
    batches = [
        (synth.make_config(flat, rows=40, base_seed=31), SamplingParams(1.0, 0, 0.95)),
        (synth.make_config(peaked, rows=12, base_seed=32), SamplingParams(0.8, 40, 0.95)),
    ]
    for call, (x_host, params) in enumerate(batches):
        x = torch.from_numpy(x_host).cuda()
        u = torch.from_numpy(synth.uniforms(x.shape[0], seed=40 + call)).cuda()
        want_ids, want_st, want_p = eng.sample(x, params, uniforms=u)
        ids, st, probs = noalloc(x, params, u)
        torch.cuda.synchronize()
        assert torch.equal(st & 0xFF, want_st & 0xFF), f"call {call}: statuses"
        assert torch.equal(ids, want_ids), f"call {call}: token ids"
        # Probabilities: identical bits (the tests' bar), within 1e-5 relative a fortiori.
        assert torch.equal(probs.view(torch.int32), want_p.view(torch.int32)), f"call {call}: probs"
