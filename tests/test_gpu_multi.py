"""Vocab-sharded sampling across GPUs: NCCL ranks, one process per GPU.

Each rank holds one vocabulary slice of the same rows; partial records are
all-gathered over NVLink and merged (rusticide_b200.sharding). Every rank must
return the tokens, statuses and probabilities that the unsharded single-GPU
call returns on the whole rows (bit for bit), and those match the oracle.
Skipped unless at least two GPUs are visible.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from rusticide_b200 import SamplingParams, synth

pytestmark = pytest.mark.gpu

ROWS, VOCAB = 64, 151936


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist
    from datetime import timedelta
    from rusticide_b200 import engine
    from rusticide_b200.sharding import VocabShardedSampler
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        x = synth.make_logits(ROWS, VOCAB, base_seed=31)
        u = synth.uniforms(ROWS, seed=8)
        params = SamplingParams(0.8, 40, 0.95)
        vs = VocabShardedSampler(engine(rank), VOCAB)
        mine = torch.from_numpy(np.ascontiguousarray(x[:, vs.offset:vs.offset + vs.width])).to(dev)
        ids, status, probs = vs.sample(mine, params, uniforms=torch.from_numpy(u).to(dev))
        torch.cuda.synchronize(dev)
        q.put((rank, ids.cpu().numpy().tolist(), status.cpu().numpy().tolist(),
               probs.cpu().numpy().view(np.uint32).tolist()))
    finally:
        dist.destroy_process_group()


LM_ROWS, LM_DIM, LM_VOCAB = 16, 1024, 32000


def _lmhead_inputs():
    """The same bf16 hidden states and LM-head weights on every rank (CPU
    generator, then moved)."""
    g = torch.Generator().manual_seed(2024)
    h = torch.randn(LM_ROWS, LM_DIM, generator=g).bfloat16()
    w = (torch.randn(LM_VOCAB, LM_DIM, generator=g) * (3.0 / LM_DIM ** 0.5)).bfloat16()
    u = torch.rand(LM_ROWS, generator=g)
    return h, w, u


def _rank_lmhead(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist
    from datetime import timedelta
    from rusticide_b200 import engine
    from rusticide_b200.sharding import VocabShardedSampler
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        h, w, u = _lmhead_inputs()
        vs = VocabShardedSampler(engine(rank), LM_VOCAB)
        w_mine = w[vs.offset:vs.offset + vs.width].contiguous().to(dev)
        ids, status, probs = vs.sample_lmhead(h.to(dev), w_mine, SamplingParams(0.8, 40, 0.95),
                                              uniforms=u.to(dev))
        torch.cuda.synchronize(dev)
        q.put((rank, ids.cpu().numpy().tolist(), status.cpu().numpy().tolist(),
               probs.cpu().numpy().view(np.uint32).tolist()))
    finally:
        dist.destroy_process_group()


def _run_ranks(target, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    while len(got) < world:
        try:
            rank, ids, st, pb = q.get(timeout=5)
            got[rank] = (ids, st, pb)
        except Exception:
            if not all(p.is_alive() or p.exitcode == 0 for p in procs):
                for p in procs:
                    if p.is_alive():
                        p.kill()
                pytest.fail("a rank failed")
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return got


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tensor_parallel_lmhead_nccl_matches_fused_call():
    """Each rank holds a vocabulary shard of the LM-head weights; the fused
    GEMM + sampler per shard, an all-gather of the shard records and the merge
    must give every rank the tokens of rsc_lmhead_sample on the whole W."""
    from rusticide_b200 import engine
    world = min(torch.cuda.device_count(), 4)
    got = _run_ranks(_rank_lmhead, world)
    h, w, u = _lmhead_inputs()
    dev = torch.device("cuda", 0)
    ids, st, pb = engine(0).lmhead_sample(h.to(dev), w.to(dev), SamplingParams(0.8, 40, 0.95),
                                          uniforms=u.to(dev))
    want = (ids.cpu().numpy().tolist(), st.cpu().numpy().tolist(),
            pb.cpu().numpy().view(np.uint32).tolist())
    for r in range(world):
        assert got[r] == want, f"rank {r}"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_vocab_sharded_nccl_matches_unsharded():
    from oracle import oracle as O
    from rusticide_b200 import engine
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    while len(got) < world:
        try:
            rank, ids, st, pb = q.get(timeout=5)
            got[rank] = (ids, st, pb)
        except Exception:
            if not all(p.is_alive() or p.exitcode == 0 for p in procs):
                for p in procs:
                    if p.is_alive():
                        p.kill()
                pytest.fail("a rank failed")
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0

    x = synth.make_logits(ROWS, VOCAB, base_seed=31)
    u = synth.uniforms(ROWS, seed=8)
    params = SamplingParams(0.8, 40, 0.95)
    dev = torch.device("cuda", 0)
    ids, st, pb = engine(0).sample(torch.from_numpy(x).to(dev), params,
                                   uniforms=torch.from_numpy(u).to(dev))
    want = (ids.cpu().numpy().tolist(), st.cpu().numpy().tolist(),
            pb.cpu().numpy().view(np.uint32).tolist())
    for r in range(world):
        assert got[r] == want, f"rank {r}"
    ref = O.sample_rows(x, O.params(0.8, 40, 0.95), u, threads=4)
    assert want[0] == [int(t) for t in ref["token"]]


PEER_ROWS, PEER_VOCAB, PEER_STEPS = 512, 151936, 3


def _peer_inputs(step):
    g = torch.Generator().manual_seed(500 + step)
    x = torch.randn(PEER_ROWS, PEER_VOCAB, generator=g) * 2.0
    u = torch.rand(PEER_ROWS, generator=g)
    return x, u


def _rank_peer(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist
    from datetime import timedelta
    from rusticide_b200 import engine
    from rusticide_b200.sharding import PeerVocabShardedSampler
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    vs = None
    try:
        vs = PeerVocabShardedSampler(engine(rank), PEER_VOCAB)
        res = []
        for step in range(PEER_STEPS):
            x, u = _peer_inputs(step)
            mine = x[:, vs.offset:vs.offset + vs.width].contiguous().to(dev)
            ids, status, probs = vs.sample(mine, SamplingParams(0.8, 40, 0.95), uniforms=u.to(dev))
            res.append((ids.cpu().numpy().tolist(), status.cpu().numpy().tolist(),
                        probs.cpu().numpy().view(np.uint32).tolist()))
        # One more step with per-row generator states (every rank merges every row).
        x, _ = _peer_inputs(PEER_STEPS)
        mine = x[:, vs.offset:vs.offset + vs.width].contiguous().to(dev)
        states = engine(rank).rng_seed(torch.arange(PEER_ROWS, dtype=torch.int64, device=dev) + 7)
        ids, status, probs = vs.sample(mine, SamplingParams(0.8, 40, 0.95), rng_states=states)
        res.append((ids.cpu().numpy().tolist(), status.cpu().numpy().tolist(),
                    probs.cpu().numpy().view(np.uint32).tolist(), states.cpu().numpy().tolist()))
        torch.cuda.synchronize(dev)
        dist.barrier()
        q.put((rank, res, None, None))
    finally:
        del vs
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_memory_vocab_sharded_matches_unsharded():
    """The records read in place over NVLink (no all-gather): three steps in a
    row (both record arrays, the step counter), every rank bit for bit equal to
    the unsharded call on the whole rows."""
    from rusticide_b200 import engine
    world = min(torch.cuda.device_count(), 4)
    got = _run_ranks(_rank_peer, world)
    dev = torch.device("cuda", 0)
    for step in range(PEER_STEPS):
        x, u = _peer_inputs(step)
        ids, st, pb = engine(0).sample(x.to(dev), SamplingParams(0.8, 40, 0.95), uniforms=u.to(dev))
        want = (ids.cpu().numpy().tolist(), st.cpu().numpy().tolist(),
                pb.cpu().numpy().view(np.uint32).tolist())
        for r in range(world):
            assert got[r][0][step] == want, f"rank {r} step {step}"
    x, _ = _peer_inputs(PEER_STEPS)
    states = engine(0).rng_seed(torch.arange(PEER_ROWS, dtype=torch.int64, device=dev) + 7)
    ids, st, pb = engine(0).sample(x.to(dev), SamplingParams(0.8, 40, 0.95), rng_states=states)
    want = (ids.cpu().numpy().tolist(), st.cpu().numpy().tolist(),
            pb.cpu().numpy().view(np.uint32).tolist(), states.cpu().numpy().tolist())
    for r in range(world):
        assert got[r][0][PEER_STEPS] == want, f"rank {r} generator-state step"
