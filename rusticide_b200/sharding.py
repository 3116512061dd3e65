"""Multi-GPU layouts of the sampler: one process per GPU.

Two ways to spread a batch over GPUs:

* row-sharded (`row_shard`): every rank samples whole rows of its own slice of
  the batch; rows are independent, so there is no collective on the data path
  (weak scaling).
* vocab-sharded (`VocabShardedSampler`): every rank holds the same rows but
  only a contiguous slice of the vocabulary, as a tensor-parallel LM head
  leaves them. Each rank reduces its slice to a fixed-size shard record per
  row (rsc_shard_partial: the slice's top-(k + tie slack) candidates in the
  total order), the records are all-gathered (NCCL over NVLink on B200), and
  every rank merges the gathered records into the same token per row
  (rsc_shard_merge). Only records cross NVLink: rows x ranks x
  rsc_shard_record_bytes(k) bytes (544 B per row and rank at k = 40)
  instead of the slices of the logits. `sample_lmhead` does the same for a
  tensor-parallel LM head: each rank's slice of the weights goes through the
  GEMM with the sampler in its epilogue (rsc_lmhead_partial), so the logits
  are never written at all.

The reference samples whole rows on one host (crates/rusticide-sampling/src/
sampler.rs:44 sample_logits, :75 greedy_logits); sharding is this
implementation's own layer on top of the same per-row result, so a sharded
batch must give the tokens of the unsharded call bit for bit.
"""

from __future__ import annotations

import time
from typing import Optional, Tuple

import torch
import torch.distributed as dist


class CollectiveError(RuntimeError):
    """The records' all-gather failed: the backend reported an error (for
    example a peer's connection closed when its process died). The process
    group has been aborted, so no later collective on it can hang; the caller
    rebuilds the group from the ranks still alive before sampling again."""


class CollectiveTimeout(CollectiveError):
    """The records' all-gather did not complete by its deadline: a rank left
    or stopped calling the sampler while its process lives on. The group has
    been aborted, as for CollectiveError."""


def _abort_group(group: Optional[dist.ProcessGroup]) -> None:
    """Ends every pending collective of `group` on this rank: the backend's
    abort where it has one (NCCL: ncclCommAbort on its communicators), else
    the group's destruction."""
    pg = group if group is not None else dist.group.WORLD
    try:
        backend = pg._get_backend(torch.device("cuda")) if torch.cuda.is_available() else None
    except Exception:
        backend = None
    if backend is not None and hasattr(backend, "abort"):
        try:
            backend.abort()
            return
        except Exception:
            pass
    try:
        dist.destroy_process_group(group)
    except Exception:
        pass


def gather_with_deadline(out: torch.Tensor, inp: torch.Tensor,
                         group: Optional[dist.ProcessGroup], timeout_s: Optional[float],
                         poll_s: float = 0.0005) -> None:
    """all_gather_into_tensor(out, inp) that gives up after timeout_s seconds.

    The collective is issued asynchronously and its completion polled from the
    host (for NCCL, is_completed() reads the collective's CUDA event, the
    counterpart of polling ncclCommGetAsyncError). Past the deadline the group
    is aborted and CollectiveTimeout raised, so a rank that never joins cannot
    hold the others forever. timeout_s None: a plain blocking all-gather
    (bounded only by the process group's own timeout)."""
    if timeout_s is None:
        dist.all_gather_into_tensor(out, inp, group=group)
        return
    rank = dist.get_rank(group)
    try:
        work = dist.all_gather_into_tensor(out, inp, group=group, async_op=True)
        deadline = time.monotonic() + timeout_s
        while not work.is_completed():
            if time.monotonic() > deadline:
                _abort_group(group)
                raise CollectiveTimeout(
                    f"shard records all-gather not complete after {timeout_s:.3f} s (rank {rank})")
            time.sleep(poll_s)
        work.wait()
    except CollectiveError:
        raise
    except RuntimeError as e:
        _abort_group(group)
        raise CollectiveError(f"shard records all-gather failed on rank {rank}: {e}") from e


def vocab_shard(vocab: int, world: int, rank: int) -> Tuple[int, int]:
    """(offset, width) of rank's vocabulary slice: equal slices of
    vocab // world columns, the last rank taking the remainder."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if vocab < world:
        raise ValueError(f"vocab {vocab} smaller than world {world}")
    base = vocab // world
    offset = rank * base
    width = vocab - offset if rank == world - 1 else base
    return offset, width


def row_shard(rows: int, world: int, rank: int) -> Tuple[int, int]:
    """(start, count) of rank's rows: the first rows % world ranks take one
    row more than the others, so counts differ by at most one."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(rows, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


class VocabShardedSampler:
    """partial -> all-gather -> merge over a process group.

    `engine` is a rusticide_b200.Engine (or any object with its
    shard_record_bytes / shard_partial / shard_merge methods). Every rank
    must call `sample` with the same rows, params and uniforms; the result
    (ids, status, probs) is the same on every rank.
    """

    def __init__(self, engine, vocab: int, group: Optional[dist.ProcessGroup] = None,
                 timeout_s: Optional[float] = None):
        """timeout_s: deadline of each records all-gather (None: wait as long
        as the process group allows); see gather_with_deadline."""
        self.engine = engine
        self.group = group
        self.timeout_s = timeout_s
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.vocab = int(vocab)
        self.offset, self.width = vocab_shard(self.vocab, self.world, self.rank)
        self._bufs: dict = {}

    def _buffers(self, rows: int, top_k: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
        key = (rows, top_k, str(device))
        if key not in self._bufs:
            rb = self.engine.shard_record_bytes(top_k)
            records = torch.empty(rows * rb, dtype=torch.uint8, device=device)
            gathered = torch.empty(self.world * rows * rb, dtype=torch.uint8, device=device)
            self._bufs = {key: (records, gathered)}
        return self._bufs[key]

    def sample(self, logits_shard: torch.Tensor, params, uniforms: Optional[torch.Tensor] = None,
               rng_states: Optional[torch.Tensor] = None, want_probs: bool = True, out=None):
        if logits_shard.dim() != 2 or logits_shard.shape[1] != self.width:
            raise ValueError(f"rank {self.rank} expects [rows, {self.width}] logits, "
                             f"got {tuple(logits_shard.shape)}")
        rows = logits_shard.shape[0]
        records, gathered = self._buffers(rows, params.top_k, logits_shard.device)
        self.engine.shard_partial(logits_shard, self.offset, self.vocab, params, records=records)
        gather_with_deadline(gathered, records, self.group, self.timeout_s)
        return self.engine.shard_merge(gathered, self.world, rows, self.vocab, params,
                                       uniforms=uniforms, rng_states=rng_states,
                                       want_probs=want_probs, out=out)

    def sample_lmhead(self, hidden: torch.Tensor, weight_shard: torch.Tensor, params,
                      uniforms: Optional[torch.Tensor] = None,
                      rng_states: Optional[torch.Tensor] = None, want_probs: bool = True,
                      out=None):
        """A tensor-parallel LM head with the sampler in its epilogue: this
        rank holds the vocabulary rows [offset, offset + width) of W
        (weight_shard, [width, dim] bf16) and every rank the same hidden
        states [rows, dim]. The shard's logits never leave the GEMM
        (rsc_lmhead_partial); only the shard records are all-gathered."""
        if weight_shard.dim() != 2 or weight_shard.shape[0] != self.width:
            raise ValueError(f"rank {self.rank} expects [{self.width}, dim] weights, "
                             f"got {tuple(weight_shard.shape)}")
        rows = hidden.shape[0]
        records, gathered = self._buffers(rows, params.top_k, hidden.device)
        self.engine.lmhead_partial(hidden, weight_shard, self.offset, self.vocab, params,
                                   records=records)
        gather_with_deadline(gathered, records, self.group, self.timeout_s)
        return self.engine.shard_merge(gathered, self.world, rows, self.vocab, params,
                                       uniforms=uniforms, rng_states=rng_states,
                                       want_probs=want_probs, out=out)


class PeerVocabShardedSampler(VocabShardedSampler):
    """The vocab-sharded step with the all-gather replaced by reads in place
    and the merge split across the ranks. Every rank's records, result arrays
    and ready words live in one symmetric allocation (every rank maps every
    other rank's copy). Per step: the partial pass writes this rank's records;
    rsc_shard_publish tells every rank they are ready; rsc_shard_merge_peers
    reads all ranks' records over NVLink (plain loads) for this rank's share of
    the rows and writes their results into every rank's result arrays;
    rsc_shard_collect waits for every share and copies the results out. Two
    record arrays and two result sets, used by step parity, keep consecutive
    steps apart (see the C header). With generator states instead of
    uniforms every rank merges every row, so that every rank advances every
    state. The result equals VocabShardedSampler's and the unsharded call's.
    Needs one warp merge per row: world * (k + 24) <= 512 and world <= 32."""

    # Byte offsets in the allocation: records-ready words, results-ready
    # words, the done counter, then the two record arrays and two result sets.
    READY_RECORDS, READY_RESULTS, COUNTER, HEAD = 0, 256, 512, 768

    def __init__(self, engine, vocab: int, group: Optional[dist.ProcessGroup] = None):
        super().__init__(engine, vocab, group)
        self._peer = None
        self._step = 0

    def _peer_state(self, rows: int, top_k: int, device):
        key = (rows, top_k, str(device))
        if self._peer is None or self._peer["key"] != key:
            import os
            # Plain peer loads and stores only: no multicast object is needed.
            os.environ.setdefault("TORCH_SYMM_MEM_DISABLE_MULTICAST", "1")
            import torch.distributed._symmetric_memory as symm
            from . import _lib
            rb = self.engine.shard_record_bytes(top_k)
            rec_span = (rows * rb + 255) // 256 * 256
            col = (rows * 4 + 255) // 256 * 256  # one result column (ids, status or probs)
            total = self.HEAD + 2 * rec_span + 2 * 3 * col
            buf = symm.empty(total, dtype=torch.uint8, device=device)
            buf.zero_()
            torch.cuda.synchronize(device)
            handle = symm.rendezvous(buf, self.group if self.group is not None else dist.group.WORLD)
            ptrs = [int(p) for p in handle.buffer_ptrs]
            if len(ptrs) != self.world:
                raise RuntimeError(f"symmetric allocation spans {len(ptrs)} ranks, not {self.world}")

            def arr(offsets):
                return torch.tensor(offsets, dtype=torch.int64, device=device)

            res0 = self.HEAD + 2 * rec_span
            sets = []
            for par in (0, 1):
                rbase = self.HEAD + par * rec_span
                obase = res0 + par * 3 * col
                sets.append({
                    "records": arr([p + rbase for p in ptrs]),
                    "ids": arr([p + obase for p in ptrs]),
                    "status": arr([p + obase + col for p in ptrs]),
                    "probs": arr([p + obase + 2 * col for p in ptrs]),
                    "rec_off": rbase, "out_off": obase,
                })
            ready_records_ptrs = arr([p + self.READY_RECORDS for p in ptrs])
            ready_results_ptrs = arr([p + self.READY_RESULTS for p in ptrs])
            # Every rank has zeroed its words before any rank publishes.
            dist.barrier(group=self.group)
            self._peer = {"key": key, "buf": buf, "handle": handle, "sets": sets, "rb": rb,
                          "col": col, "ready_records_ptrs": ready_records_ptrs,
                          "ready_results_ptrs": ready_results_ptrs, "lib": _lib}
            self._step = 0
        return self._peer

    def sample(self, logits_shard: torch.Tensor, params, uniforms: Optional[torch.Tensor] = None,
               rng_states: Optional[torch.Tensor] = None, want_probs: bool = True, out=None):
        if logits_shard.dim() != 2 or logits_shard.shape[1] != self.width:
            raise ValueError(f"rank {self.rank} expects [rows, {self.width}] logits, "
                             f"got {tuple(logits_shard.shape)}")
        rows = logits_shard.shape[0]
        st = self._peer_state(rows, params.top_k, logits_shard.device)
        self._step += 1
        step, par = self._step, self._step & 1
        cur = st["sets"][par]
        buf, base = st["buf"], st["buf"].data_ptr()
        mine = buf[cur["rec_off"]:cur["rec_off"] + rows * st["rb"]]
        self.engine.shard_partial(logits_shard, self.offset, self.vocab, params, records=mine)
        self.engine.shard_publish(st["ready_records_ptrs"], self.world, self.rank, step)
        share = rng_states is None
        x = st["lib"].RscPeerExchange(
            cur["records"].data_ptr(), base + self.READY_RECORDS,
            st["ready_results_ptrs"].data_ptr() if share else None, base + self.COUNTER,
            cur["ids"].data_ptr(), cur["status"].data_ptr(),
            cur["probs"].data_ptr() if want_probs else None)
        self.engine.shard_merge_peers(x, step, self.world, self.rank, rows, self.vocab, params,
                                      uniforms=uniforms, rng_states=rng_states)
        out = out if out is not None else self.engine._outputs(rows, want_probs)
        ids_addr = base + cur["out_off"]
        if share:
            return self.engine.shard_collect(base + self.READY_RESULTS, step, self.world, rows,
                                             ids_addr, ids_addr + st["col"],
                                             ids_addr + 2 * st["col"] if want_probs else None, out)
        # Every row was merged here: this rank's result arrays hold them all.
        oi, os_, op = out
        col = st["col"]
        oi.copy_(buf[cur["out_off"]:cur["out_off"] + rows * 4].view(torch.int32))
        os_.copy_(buf[cur["out_off"] + col:cur["out_off"] + col + rows * 4].view(torch.int32))
        if op is not None:
            op.copy_(buf[cur["out_off"] + 2 * col:cur["out_off"] + 2 * col + rows * 4]
                     .view(torch.float32))
        return out
