"""Host logic of the multi-GPU layouts, on CPU with gloo ranks.

The vocab-sharded orchestration (rusticide_b200.sharding.VocabShardedSampler:
partial -> all-gather -> merge) runs here over a world of 2 and 3 gloo ranks
with a stand-in engine whose "records" carry the shard's raw columns and whose
merge reassembles the rows and samples them with the oracle. That pins what
the host layer owns: every rank's slice bounds, the order of the gathered
records, and the same result on every rank, against the oracle on the
unsharded rows (crates/rusticide-sampling/src/sampler.rs:44). The device
records and their merge are covered by the GPU parity tests.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rusticide_b200 import SamplingParams, synth
from rusticide_b200.sharding import (CollectiveError, CollectiveTimeout, VocabShardedSampler,
                                     row_shard, vocab_shard)


def test_vocab_shard_covers_the_vocabulary():
    for vocab in (7, 32000, 151936, 151937):
        for world in (1, 2, 3, 4, 7, 8):
            if vocab < world:
                continue
            spans = [vocab_shard(vocab, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (o0, w0), (o1, _) in zip(spans, spans[1:]):
                assert o0 + w0 == o1
            assert spans[-1][0] + spans[-1][1] == vocab
            assert all(w >= vocab // world for _, w in spans)
    with pytest.raises(ValueError):
        vocab_shard(3, 4, 0)
    with pytest.raises(ValueError):
        vocab_shard(100, 2, 2)


def test_row_shard_balances_rows():
    for rows in (0, 1, 5, 1024, 1027):
        for world in (1, 2, 3, 8):
            spans = [row_shard(rows, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (s0, c0), (s1, _) in zip(spans, spans[1:]):
                assert s0 + c0 == s1
            assert sum(c for _, c in spans) == rows
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1


class _ColumnsEngine:
    """Stand-in engine: a record is (offset, width) + the shard's columns."""

    def __init__(self, max_width: int):
        self.max_width = max_width

    def shard_record_bytes(self, top_k: int) -> int:
        return 8 + 4 * self.max_width

    def shard_partial(self, logits, offset, vocab, params, records):
        rows, width = logits.shape
        rb = self.shard_record_bytes(params.top_k)
        rec = records.view(rows, rb)
        for r in range(rows):
            head = np.array([offset, width], dtype=np.int32).view(np.uint8)
            body = np.zeros(self.max_width, dtype=np.float32)
            body[:width] = logits[r].numpy()
            rec[r, :8] = torch.from_numpy(head.copy())
            rec[r, 8:] = torch.from_numpy(body.view(np.uint8).copy())
        return records

    def shard_merge(self, gathered, n_shards, rows, vocab, params, uniforms=None,
                    rng_states=None, want_probs=True, out=None):
        from oracle import oracle as O
        rb = self.shard_record_bytes(params.top_k)
        g = gathered.view(n_shards, rows, rb).numpy()
        full = np.full((rows, vocab), np.nan, dtype=np.float32)
        for s in range(n_shards):
            for r in range(rows):
                off, width = g[s, r, :8].view(np.int32)
                full[r, off:off + width] = g[s, r, 8:8 + 4 * width].view(np.float32)
        assert not np.isnan(full).any(), "gathered records leave columns uncovered"
        op = O.params(params.temperature, params.top_k, params.top_p)
        return O.sample_rows(full, op, uniforms.numpy(), threads=1)


class _LmheadColumnsEngine(_ColumnsEngine):
    """Stand-in engine for the sharded LM head: the shard's logits are the f32
    product of its weight rows with the hidden states, then a columns record."""

    def lmhead_partial(self, hidden, weight_shard, offset, vocab, params, records):
        logits = (hidden.float() @ weight_shard.float().T).contiguous()
        return self.shard_partial(logits, offset, vocab, params, records)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, rows, vocab, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = synth.make_logits(rows, vocab, base_seed=77)
        u = torch.from_numpy(synth.uniforms(rows, seed=5))
        params = SamplingParams(0.8, 40, 0.95)
        eng = _ColumnsEngine(max_width=vocab // world + vocab % world)
        vs = VocabShardedSampler(eng, vocab)
        mine = torch.from_numpy(np.ascontiguousarray(x[:, vs.offset:vs.offset + vs.width]))
        res = vs.sample(mine, params, uniforms=u)
        q.put((rank, [(int(t), int(st)) for t, st in zip(res["token"], res["status"])]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_vocab_sharded_orchestration_matches_unsharded(world):
    from oracle import oracle as O
    rows, vocab = 6, 1001
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, rows, vocab, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    while len(got) < world:
        try:
            rank, res = q.get(timeout=5)
            got[rank] = res
        except Exception:
            assert all(p.is_alive() or p.exitcode == 0 for p in procs), "a rank failed"
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    x = synth.make_logits(rows, vocab, base_seed=77)
    u = synth.uniforms(rows, seed=5)
    ref = O.sample_rows(x, O.params(0.8, 40, 0.95), u, threads=1)
    want = [(int(t), int(st)) for t, st in zip(ref["token"], ref["status"])]
    for r in range(world):
        assert got[r] == want, f"rank {r}"


def _rank_lmhead_main(rank, world, port, rows, dim, vocab, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(9)
        h = torch.randn(rows, dim, generator=g).bfloat16()
        w = torch.randn(vocab, dim, generator=g).bfloat16()
        u = torch.from_numpy(synth.uniforms(rows, seed=6))
        eng = _LmheadColumnsEngine(max_width=vocab // world + vocab % world)
        vs = VocabShardedSampler(eng, vocab)
        with pytest.raises(ValueError):
            vs.sample_lmhead(h, w, SamplingParams(0.8, 40, 0.95), uniforms=u)  # not a shard
        res = vs.sample_lmhead(h, w[vs.offset:vs.offset + vs.width], SamplingParams(0.8, 40, 0.95),
                               uniforms=u)
        q.put((rank, [(int(t), int(st)) for t, st in zip(res["token"], res["status"])]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_lmhead_orchestration_matches_unsharded(world):
    """VocabShardedSampler.sample_lmhead: each rank's weight rows, its global
    offsets and the gathered order give the oracle's tokens on the whole
    product (the device GEMM and records are covered by the GPU tests)."""
    from oracle import oracle as O
    rows, dim, vocab = 5, 16, 1001
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_lmhead_main, args=(r, world, port, rows, dim, vocab, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    while len(got) < world:
        try:
            rank, res = q.get(timeout=5)
            got[rank] = res
        except Exception:
            assert all(p.is_alive() or p.exitcode == 0 for p in procs), "a rank failed"
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(9)
    h = torch.randn(rows, dim, generator=g).bfloat16()
    w = torch.randn(vocab, dim, generator=g).bfloat16()
    x = (h.float() @ w.float().T).numpy()
    u = synth.uniforms(rows, seed=6)
    ref = O.sample_rows(x, O.params(0.8, 40, 0.95), u, threads=1)
    want = [(int(t), int(st)) for t, st in zip(ref["token"], ref["status"])]
    for r in range(world):
        assert got[r] == want, f"rank {r}"


def _rank_dropout_main(rank, world, port, rows, vocab, mode, q):
    """Rank 0 samples with a short all-gather deadline. The other ranks leave
    between steps without joining the collective: mode "stall" keeps their
    process alive (a rank stuck elsewhere), mode "exit" ends it (a rank that
    died)."""
    import time as _t
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    if rank != 0:
        q.put((rank, "left"))
        if mode == "stall":
            _t.sleep(5.0)
        return  # no collective, no destroy: this rank is gone
    x = synth.make_logits(rows, vocab, base_seed=77)
    u = torch.from_numpy(synth.uniforms(rows, seed=5))
    eng = _ColumnsEngine(max_width=vocab // world + vocab % world)
    vs = VocabShardedSampler(eng, vocab, timeout_s=0.5)
    mine = torch.from_numpy(np.ascontiguousarray(x[:, vs.offset:vs.offset + vs.width]))
    t0 = _t.monotonic()
    try:
        vs.sample(mine, SamplingParams(0.8, 40, 0.95), uniforms=u)
        q.put((0, ("no error", 0.0)))
    except CollectiveTimeout:
        q.put((0, ("timeout", _t.monotonic() - t0)))
    except CollectiveError:
        q.put((0, ("error", _t.monotonic() - t0)))


@pytest.mark.parametrize("mode", ["stall", "exit"])
def test_vocab_sharded_rank_dropout_is_detected(mode):
    """Failure detection on the host: a rank that never joins the records'
    all-gather makes the others raise instead of waiting for ever:
    CollectiveTimeout after the deadline while its process lives, or
    CollectiveError (or the timeout) once its connection has closed; the group
    is aborted in both cases."""
    world, rows, vocab = 2, 4, 501
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_dropout_main, args=(r, world, port, rows, vocab, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        while len(got) < world:
            rank, res = q.get(timeout=60)
            got[rank] = res
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert got[1] == "left"
    kind, secs = got[0]
    if mode == "stall":
        assert kind == "timeout", got[0]
        assert 0.4 < secs < 20.0
    else:
        assert kind in ("timeout", "error"), got[0]
        assert secs < 20.0
