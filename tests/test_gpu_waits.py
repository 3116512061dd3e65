"""Bounded device waits, made to run out on purpose (failure detection without
a GPU fault).

Every spin in the kernels gives up after the library's wait limit (2 s of the
GPU's global timer) and reports RSC_ROW_INTERNAL for the row it was serving,
instead of hanging the device. Here the wait is the streaming kernel's lock on
a scratch slot, which a row takes only when its candidate list overflows with
ties and it must be finished by the large-row code. rsc_debug_hold_scratch
marks every slot taken, so nothing will ever release the lock the row waits
for: no bulk copy is in flight during that wait, and no memory is touched out
of bounds. The row must come back RSC_ROW_INTERNAL after about the limit, the
other rows of the same call must be exact, and after the slots are released
the same call must sample every row exactly again (the context survived).
"""

import time

import numpy as np
import pytest
import torch

from oracle import oracle as O
from rusticide_b200 import SamplingParams, synth
from rusticide_b200._lib import RSC_ROW_INTERNAL
from rusticide_b200.sampler import Engine

pytestmark = pytest.mark.gpu


def _rows():
    vocab = 20000
    x = synth.make_logits(4, vocab, base_seed=21, dist="peaked", spikes=(5, 20))
    rng = np.random.default_rng(3)
    x[2] = rng.integers(0, 4, vocab).astype(np.float32)  # 4 values: thousands tied at the top
    return x


def test_slot_wait_runs_out_and_reports_internal():
    x = _rows()
    u = synth.uniforms(x.shape[0], seed=9)
    params = SamplingParams(0.8, 40, 0.95)
    want = O.sample_rows(x, O.params(0.8, 40, 0.95), u)
    eng = Engine(0, max_rows=x.shape[0], max_vocab=x.shape[1])
    try:
        xd = torch.from_numpy(x).cuda()
        ud = torch.from_numpy(u).cuda()
        # Free slots: every row exact.
        ids, st, _ = eng.sample(xd, params, uniforms=ud)
        torch.cuda.synchronize()
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), want["token"])
        assert np.array_equal(st.cpu().numpy() & 0xFF, want["status"])
        # Held slots: the tie row's wait runs out.
        eng.hold_scratch(True)
        t0 = time.monotonic()
        ids, st, _ = eng.sample(xd, params, uniforms=ud)
        torch.cuda.synchronize()
        waited = time.monotonic() - t0
        st = st.cpu().numpy()
        got = ids.cpu().numpy().view(np.uint32)
        assert st[2] & 0xFF == RSC_ROW_INTERNAL, st
        assert 1.0 < waited < 30.0, waited
        others = [r for r in range(x.shape[0]) if r != 2]
        assert np.array_equal(got[others], want["token"][others])
        assert np.array_equal(st[others] & 0xFF, want["status"][others])
        # Released: the device and the handle still work, every row exact.
        eng.hold_scratch(False)
        ids, st, _ = eng.sample(xd, params, uniforms=ud)
        torch.cuda.synchronize()
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), want["token"])
        assert np.array_equal(st.cpu().numpy() & 0xFF, want["status"])
    finally:
        eng.close()
