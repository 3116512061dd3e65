"""Host-side mirror of rusticide-sampling's public API over the CUDA engine.

`Sampler`, `SamplingParams` and the `SamplingError` family keep the names,
argument meaning and error behaviour of the Rust crate
(crates/rusticide-sampling/src/{sampler,params,error,logits}.rs), so that code
written against the reference reads the same here. Every call runs on the GPU
through the C ABI of librusticide_cuda.so; there is no CPU fallback.

`Engine` is the batched form the engine exists for: one call samples R rows of
an R x V logit matrix already in device memory.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import RscParams, check


# ---------------------------------------------------------------------------
# SamplingParams, crates/rusticide-sampling/src/params.rs:5-22
# ---------------------------------------------------------------------------
@dataclass
class SamplingParams:
    temperature: float = 0.8
    top_k: int = 40
    top_p: float = 0.9
    repetition_penalty: float = 1.0
    seed: int = 0

    def to_c(self) -> RscParams:
        return RscParams(float(self.temperature), int(self.top_k) & 0xFFFFFFFF, float(self.top_p),
                         float(self.repetition_penalty), int(self.seed) & 0xFFFFFFFFFFFFFFFF)


# ---------------------------------------------------------------------------
# SamplingError, crates/rusticide-sampling/src/error.rs:5-15
# ---------------------------------------------------------------------------
class SamplingError(Exception):
    """Base of the sampler's errors."""


class TensorError(SamplingError):
    """SamplingError::Tensor: the logits tensor is not f32."""

    def __init__(self, expected: str, got: str):
        super().__init__(f"tensor error: dtype mismatch: expected {expected}, got {got}")
        self.expected = expected
        self.got = got


class InvalidShape(SamplingError):
    """SamplingError::InvalidShape: logits are neither [V] nor [1, V]."""

    def __init__(self, dims: Sequence[int]):
        super().__init__(f"logits tensor has wrong shape: expected 1D or 2D, got {list(dims)}")
        self.dims = list(dims)


class NoValidTokens(SamplingError):
    """SamplingError::NoValidTokens."""

    def __init__(self):
        super().__init__("all logits are -inf or NaN after filtering")


class VocabOverflow(SamplingError):
    """SamplingError::VocabOverflow."""

    def __init__(self):
        super().__init__("vocabulary size exceeds u32 range")


def row_error(status: int) -> Optional[SamplingError]:
    """Maps a per-row status word to the reference's error, or None for OK."""
    code = int(status) & 0xFF
    if code == _lib.RSC_ROW_OK:
        return None
    if code == _lib.RSC_ROW_NO_VALID_TOKENS:
        return NoValidTokens()
    if code == _lib.RSC_ROW_VOCAB_OVERFLOW:
        return VocabOverflow()
    raise RuntimeError(f"row not sampled: device status {int(status):#x}")


def extract_logits(t: torch.Tensor) -> torch.Tensor:
    """extract_logits, crates/rusticide-sampling/src/logits.rs:9-23: accepts f32
    tensors of shape [V] or [1, V] and returns the row. (The NaN -> -inf
    rewrite of the reference happens on the device.)"""
    dims = list(t.shape)
    if not (len(dims) == 1 or (len(dims) == 2 and dims[0] == 1)):
        raise InvalidShape(dims)
    if t.dtype != torch.float32:
        raise TensorError("F32", str(t.dtype).replace("torch.", "").upper())
    return t.reshape(-1)


def _u64_to_i64(x: int) -> int:
    x &= 0xFFFFFFFFFFFFFFFF
    return x - (1 << 64) if x >= (1 << 63) else x


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ---------------------------------------------------------------------------
# Engine: one rsc_sampler handle per device, grown on demand.
# ---------------------------------------------------------------------------
class Engine:
    """Batched sampling on one GPU through the C ABI."""

    def __init__(self, device: int | torch.device | None = None, max_rows: int = 1,
                 max_vocab: int = 1):
        if not torch.cuda.is_available():
            raise RuntimeError("rusticide_b200 needs a CUDA device; there is no CPU fallback")
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if dev.type != "cuda":
            dev = torch.device("cuda", dev.index or 0)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.lib = _lib.lib()
        self._h = ctypes.c_void_p()
        self.max_rows = 0
        self.max_vocab = 0
        self._create(max(1, max_rows), max(1, max_vocab))

    def _create(self, rows: int, vocab: int) -> None:
        if self._h:
            torch.cuda.synchronize(self.device)
            check(self.lib.rsc_sampler_destroy(self._h), "rsc_sampler_destroy")
            self._h = ctypes.c_void_p()
        h = ctypes.c_void_p()
        check(self.lib.rsc_sampler_create(self.device.index, rows, vocab, ctypes.byref(h)),
              "rsc_sampler_create")
        self._h = h
        self.max_rows, self.max_vocab = rows, vocab

    def ensure(self, rows: int, vocab: int) -> None:
        if rows > self.max_rows or vocab > self.max_vocab:
            self._create(max(rows, self.max_rows), max(vocab, self.max_vocab))

    def close(self) -> None:
        if self._h:
            torch.cuda.synchronize(self.device)
            self.lib.rsc_sampler_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def launch_count(self) -> int:
        return int(self.lib.rsc_launch_count(self._h))

    def hold_scratch(self, hold: bool) -> None:
        """rsc_debug_hold_scratch: marks the handle's scratch slots taken (or
        free) on the current stream, so that a row needing one exercises the
        bounded wait and reports RSC_ROW_INTERNAL. Test hook only."""
        check(self.lib.rsc_debug_hold_scratch(self._h, 1 if hold else 0,
                                               _stream_ptr(self.device)),
              "rsc_debug_hold_scratch")

    # -- helpers --------------------------------------------------------------
    def _check_rows(self, logits: torch.Tensor) -> tuple[int, int, int]:
        if logits.device != self.device:
            raise ValueError(f"logits on {logits.device}, engine on {self.device}")
        if logits.dtype != torch.float32:
            raise TensorError("F32", str(logits.dtype).replace("torch.", "").upper())
        if logits.dim() != 2:
            raise InvalidShape(list(logits.shape))
        rows, vocab = logits.shape
        stride = logits.stride(0) if rows > 1 else vocab
        if rows > 0 and vocab > 0 and logits.stride(1) != 1:
            raise ValueError("logit rows must be contiguous")
        self.ensure(rows, vocab)
        return rows, vocab, stride

    def _outputs(self, rows: int, want_probs: bool):
        ids = torch.empty(rows, dtype=torch.int32, device=self.device)
        status = torch.empty(rows, dtype=torch.int32, device=self.device)
        probs = torch.empty(rows, dtype=torch.float32, device=self.device) if want_probs else None
        return ids, status, probs

    # -- batched calls --------------------------------------------------------
    def sample(self, logits: torch.Tensor, params: SamplingParams,
               uniforms: Optional[torch.Tensor] = None, rng_states: Optional[torch.Tensor] = None,
               want_probs: bool = True, out=None):
        """rsc_sample: batched Sampler::sample_logits. Returns (ids, status, probs)."""
        rows, vocab, stride = self._check_rows(logits)
        ids, status, probs = out if out is not None else self._outputs(rows, want_probs)
        c = params.to_c()
        check(self.lib.rsc_sample(self._h, logits.data_ptr(), rows, vocab, stride, ctypes.byref(c),
                                  _ptr(uniforms), _ptr(rng_states), ids.data_ptr(),
                                  status.data_ptr(), _ptr(probs), _stream_ptr(self.device)),
              "rsc_sample")
        return ids, status, probs

    def sample_rows(self, logits: torch.Tensor, params: Sequence[SamplingParams],
                    uniforms: Optional[torch.Tensor] = None,
                    rng_states: Optional[torch.Tensor] = None, want_probs: bool = True, out=None):
        """rsc_sample_rows: row r is Sampler::sample_logits(row r, params[r]).
        Returns (ids, status, probs)."""
        rows, vocab, stride = self._check_rows(logits)
        if len(params) != rows:
            raise SamplingError(f"InvalidShape: {len(params)} parameter sets for {rows} rows")
        ids, status, probs = out if out is not None else self._outputs(rows, want_probs)
        arr = (_lib.RscParams * max(1, rows))(*[p.to_c() for p in params])
        check(self.lib.rsc_sample_rows(self._h, logits.data_ptr(), rows, vocab, stride, arr,
                                       _ptr(uniforms), _ptr(rng_states), ids.data_ptr(),
                                       status.data_ptr(), _ptr(probs), _stream_ptr(self.device)),
              "rsc_sample_rows")
        return ids, status, probs

    def sample_ex(self, logits: torch.Tensor, params: SamplingParams,
                  uniforms: Optional[torch.Tensor] = None,
                  rng_states: Optional[torch.Tensor] = None, survivor_cap: int = 0,
                  logprobs: bool = False):
        """rsc_sample_ex: rsc_sample plus each row's surviving candidate set and
        its probabilities. Returns (ids, status, probs, n_survivors,
        survivor_ids[rows, cap], survivor_probs[rows, cap]); with logprobs,
        also (row_logsumexp, token_logprob, survivor_logprobs[rows, cap]):
        log-probabilities over the whole row of scaled logits."""
        rows, vocab, stride = self._check_rows(logits)
        ids, status, probs = self._outputs(rows, True)
        nsurv = torch.empty(rows, dtype=torch.int32, device=self.device)
        cap = max(1, int(survivor_cap))
        surv = torch.full((rows, cap), -1, dtype=torch.int32, device=self.device)
        survp = torch.full((rows, cap), float("nan"), dtype=torch.float32, device=self.device)
        lse = tok_lp = surv_lp = None
        if logprobs:
            lse = torch.full((rows,), float("nan"), dtype=torch.float32, device=self.device)
            tok_lp = torch.full((rows,), float("nan"), dtype=torch.float32, device=self.device)
            surv_lp = torch.full((rows, cap), float("nan"), dtype=torch.float32, device=self.device)
        ex = _lib.RscSampleExtras(nsurv.data_ptr(), surv.data_ptr() if survivor_cap else None,
                                  cap if survivor_cap else 0,
                                  survp.data_ptr() if survivor_cap else None,
                                  _ptr(lse), _ptr(tok_lp),
                                  surv_lp.data_ptr() if (logprobs and survivor_cap) else None)
        c = params.to_c()
        check(self.lib.rsc_sample_ex(self._h, logits.data_ptr(), rows, vocab, stride,
                                     ctypes.byref(c), _ptr(uniforms), _ptr(rng_states),
                                     ids.data_ptr(), status.data_ptr(), _ptr(probs),
                                     ctypes.byref(ex), _stream_ptr(self.device)), "rsc_sample_ex")
        if logprobs:
            return ids, status, probs, nsurv, surv, survp, lse, tok_lp, surv_lp
        return ids, status, probs, nsurv, surv, survp

    def pick(self, logits: torch.Tensor, params: SamplingParams,
             uniforms: Optional[torch.Tensor] = None, rng_states: Optional[torch.Tensor] = None,
             want_probs: bool = True, out=None):
        """rsc_pick: generate.rs:117-124 over a batch."""
        rows, vocab, stride = self._check_rows(logits)
        ids, status, probs = out if out is not None else self._outputs(rows, want_probs)
        c = params.to_c()
        check(self.lib.rsc_pick(self._h, logits.data_ptr(), rows, vocab, stride, ctypes.byref(c),
                                _ptr(uniforms), _ptr(rng_states), ids.data_ptr(),
                                status.data_ptr(), _ptr(probs), _stream_ptr(self.device)),
              "rsc_pick")
        return ids, status, probs

    def greedy(self, logits: torch.Tensor, out=None):
        """rsc_greedy: batched Sampler::greedy_logits. Returns (ids, status)."""
        rows, vocab, stride = self._check_rows(logits)
        ids, status, _ = out if out is not None else self._outputs(rows, False)
        check(self.lib.rsc_greedy(self._h, logits.data_ptr(), rows, vocab, stride, ids.data_ptr(),
                                  status.data_ptr(), _stream_ptr(self.device)), "rsc_greedy")
        return ids, status

    def sample_with_temp(self, logits: torch.Tensor, temperature: float,
                         uniforms: Optional[torch.Tensor] = None,
                         rng_states: Optional[torch.Tensor] = None, want_probs: bool = True):
        """rsc_sample_with_temp: batched Sampler::sample_with_temp."""
        rows, vocab, stride = self._check_rows(logits)
        ids, status, probs = self._outputs(rows, want_probs)
        check(self.lib.rsc_sample_with_temp(self._h, logits.data_ptr(), rows, vocab, stride,
                                            float(temperature), _ptr(uniforms), _ptr(rng_states),
                                            ids.data_ptr(), status.data_ptr(), _ptr(probs),
                                            _stream_ptr(self.device)), "rsc_sample_with_temp")
        return ids, status, probs

    def penalize(self, logits: torch.Tensor, tokens: torch.Tensor, penalty: float) -> None:
        """rsc_penalize: apply_repetition_penalty on every row, in place."""
        rows, vocab, stride = self._check_rows(logits)
        tokens = tokens.to(device=self.device, dtype=torch.int32).contiguous()
        check(self.lib.rsc_penalize(self._h, logits.data_ptr(), rows, vocab, stride,
                                    tokens.data_ptr(), tokens.numel(), float(penalty),
                                    _stream_ptr(self.device)), "rsc_penalize")

    def rng_seed(self, seeds: torch.Tensor) -> torch.Tensor:
        """rsc_rng_seed: per-row generator states from u64 seeds (int64 storage)."""
        seeds = seeds.to(device=self.device, dtype=torch.int64).contiguous()
        states = torch.empty_like(seeds)
        check(self.lib.rsc_rng_seed(seeds.data_ptr(), states.data_ptr(), seeds.numel(),
                                    _stream_ptr(self.device)), "rsc_rng_seed")
        return states

    def pick_host(self, logits, params: SamplingParams, uniforms=None):
        """rsc_pick_host: host (numpy or CPU tensor) logits in, host results out."""
        import numpy as np
        x = np.ascontiguousarray(logits, dtype=np.float32)
        if x.ndim == 1:
            x = x[None, :]
        rows, vocab = x.shape
        self.ensure(rows, vocab)
        u = None if uniforms is None else np.ascontiguousarray(uniforms, dtype=np.float32)
        ids = np.empty(rows, dtype=np.uint32)
        status = np.empty(rows, dtype=np.int32)
        probs = np.empty(rows, dtype=np.float32)
        c = params.to_c()
        check(self.lib.rsc_pick_host(self._h, x.ctypes.data, rows, vocab, ctypes.byref(c),
                                     None if u is None else u.ctypes.data, ids.ctypes.data,
                                     status.ctypes.data, probs.ctypes.data), "rsc_pick_host")
        return ids, status, probs

    # -- vocab-sharded mode ---------------------------------------------------
    def shard_record_bytes(self, top_k: int) -> int:
        return int(self.lib.rsc_shard_record_bytes(int(top_k)))

    def shard_partial(self, logits: torch.Tensor, shard_offset: int, global_vocab: int,
                      params: SamplingParams, records: Optional[torch.Tensor] = None) -> torch.Tensor:
        rows, vocab, stride = self._check_rows(logits)
        rb = self.shard_record_bytes(params.top_k)
        if records is None:
            records = torch.empty(rows * rb, dtype=torch.uint8, device=self.device)
        c = params.to_c()
        check(self.lib.rsc_shard_partial(self._h, logits.data_ptr(), rows, vocab, stride,
                                         int(shard_offset), int(global_vocab), ctypes.byref(c),
                                         records.data_ptr(), _stream_ptr(self.device)),
              "rsc_shard_partial")
        return records

    def shard_publish(self, ready_ptrs: torch.Tensor, n_shards: int, my_shard: int, step: int) -> None:
        """rsc_shard_publish: `step` into word my_shard of every rank's ready
        array (ready_ptrs: int64 device tensor of the ranks' ready arrays)."""
        check(self.lib.rsc_shard_publish(ready_ptrs.data_ptr(), int(n_shards), int(my_shard),
                                         int(step) & 0xFFFFFFFF, _stream_ptr(self.device)),
              "rsc_shard_publish")

    def shard_merge_peers(self, exchange, step: int, n_shards: int, my_shard: int, rows: int,
                          global_vocab: int, params: SamplingParams,
                          uniforms: Optional[torch.Tensor] = None,
                          rng_states: Optional[torch.Tensor] = None) -> None:
        """rsc_shard_merge_peers (exchange: an _lib.RscPeerExchange of device
        addresses); the results land in the exchange's result arrays."""
        self.ensure(rows, 1)
        c = params.to_c()
        check(self.lib.rsc_shard_merge_peers(self._h, ctypes.byref(exchange), int(step) & 0xFFFFFFFF,
                                             int(n_shards), int(my_shard), rows, int(global_vocab),
                                             ctypes.byref(c), _ptr(uniforms), _ptr(rng_states),
                                             _stream_ptr(self.device)),
              "rsc_shard_merge_peers")

    def shard_collect(self, ready_results: int, step: int, n_shards: int, rows: int, ids: int,
                      status: int, probs: Optional[int], out):
        """rsc_shard_collect: waits for every rank's results of `step`, then
        copies this rank's result arrays (device addresses) into `out`."""
        oi, os_, op = out
        check(self.lib.rsc_shard_collect(int(ready_results), int(step) & 0xFFFFFFFF, int(n_shards),
                                         rows, int(ids), int(status), probs, oi.data_ptr(),
                                         os_.data_ptr(), _ptr(op), _stream_ptr(self.device)),
              "rsc_shard_collect")
        return out

    def shard_merge(self, gathered: torch.Tensor, n_shards: int, rows: int, global_vocab: int,
                    params: SamplingParams, uniforms: Optional[torch.Tensor] = None,
                    rng_states: Optional[torch.Tensor] = None, want_probs: bool = True, out=None):
        self.ensure(rows, 1)
        ids, status, probs = out if out is not None else self._outputs(rows, want_probs)
        c = params.to_c()
        check(self.lib.rsc_shard_merge(self._h, gathered.data_ptr(), int(n_shards), rows,
                                       int(global_vocab), ctypes.byref(c), _ptr(uniforms),
                                       _ptr(rng_states), ids.data_ptr(), status.data_ptr(),
                                       _ptr(probs), _stream_ptr(self.device)), "rsc_shard_merge")
        return ids, status, probs

    # -- LM head with the sampler fused into its epilogue ----------------------
    @staticmethod
    def _lmhead_args(hidden: torch.Tensor, weight: torch.Tensor):
        if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
            raise TensorError("bf16", f"{hidden.dtype}/{weight.dtype}")
        if hidden.dim() != 2 or weight.dim() != 2 or hidden.shape[1] != weight.shape[1]:
            raise InvalidShape(list(hidden.shape) + list(weight.shape))
        return hidden.contiguous(), weight.contiguous()

    def lmhead_logits(self, hidden: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        """hidden . weight^T in f32 (bf16 inputs) on the tensor cores."""
        hidden, weight = self._lmhead_args(hidden, weight)
        rows, dim = hidden.shape
        vocab = weight.shape[0]
        self.ensure(rows, 1)
        out = torch.empty((rows, vocab), dtype=torch.float32, device=self.device)
        check(self.lib.rsc_lmhead_logits(self._h, hidden.data_ptr(), weight.data_ptr(), rows, dim,
                                         vocab, out.data_ptr(), _stream_ptr(self.device)),
              "rsc_lmhead_logits")
        return out

    def lmhead_sample(self, hidden: torch.Tensor, weight: torch.Tensor, params: SamplingParams,
                      uniforms: Optional[torch.Tensor] = None,
                      rng_states: Optional[torch.Tensor] = None, want_probs: bool = True,
                      out=None):
        """sample(hidden . weight^T) without writing the logits."""
        hidden, weight = self._lmhead_args(hidden, weight)
        rows, dim = hidden.shape
        vocab = weight.shape[0]
        self.ensure(rows, 1)
        ids, status, probs = out if out is not None else self._outputs(rows, want_probs)
        c = params.to_c()
        check(self.lib.rsc_lmhead_sample(self._h, hidden.data_ptr(), weight.data_ptr(), rows, dim,
                                         vocab, ctypes.byref(c), _ptr(uniforms), _ptr(rng_states),
                                         ids.data_ptr(), status.data_ptr(), _ptr(probs),
                                         _stream_ptr(self.device)), "rsc_lmhead_sample")
        return ids, status, probs

    def lmhead_partial(self, hidden: torch.Tensor, weight_shard: torch.Tensor, shard_offset: int,
                       global_vocab: int, params: SamplingParams,
                       records: Optional[torch.Tensor] = None) -> torch.Tensor:
        """rsc_lmhead_partial: this rank's shard record per row for a
        vocabulary shard of the LM head (rows [shard_offset, shard_offset +
        weight_shard.shape[0]) of W), to all-gather and pass to shard_merge."""
        hidden, weight_shard = self._lmhead_args(hidden, weight_shard)
        rows, dim = hidden.shape
        self.ensure(rows, 1)
        rb = self.shard_record_bytes(params.top_k)
        if records is None:
            records = torch.empty(rows * rb, dtype=torch.uint8, device=self.device)
        c = params.to_c()
        check(self.lib.rsc_lmhead_partial(self._h, hidden.data_ptr(), weight_shard.data_ptr(), rows,
                                          dim, weight_shard.shape[0], int(shard_offset),
                                          int(global_vocab), ctypes.byref(c), records.data_ptr(),
                                          _stream_ptr(self.device)), "rsc_lmhead_partial")
        return records


_ENGINES: dict[int, Engine] = {}


def engine(device: int | torch.device | None = None) -> Engine:
    """The shared Engine of a device."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _ENGINES:
        _ENGINES[idx] = Engine(idx)
    return _ENGINES[idx]


# ---------------------------------------------------------------------------
# Sampler, crates/rusticide-sampling/src/sampler.rs:13-139
# ---------------------------------------------------------------------------
class Sampler:
    """One generation stream's sampler: a seeded generator plus the sampling
    entry points of the reference, evaluated on the GPU.

    The generator state lives on the device and advances only when a call
    consumes a draw (src/sampler.rs:112), like the reference's rng."""

    def __init__(self, seed: int, device: int | torch.device | None = None):
        self._engine = engine(device)
        self.device = self._engine.device
        seeds = torch.tensor([_u64_to_i64(seed)], dtype=torch.int64, device=self.device)
        self._state = self._engine.rng_seed(seeds)

    @classmethod
    def new(cls, seed: int, device=None) -> "Sampler":
        return cls(seed, device)

    def _row(self, logits) -> torch.Tensor:
        if not isinstance(logits, torch.Tensor):
            logits = torch.tensor(list(logits), dtype=torch.float32)
        if logits.dtype != torch.float32:
            raise TensorError("F32", str(logits.dtype).replace("torch.", "").upper())
        return logits.reshape(1, -1).to(self.device)

    @staticmethod
    def _result(ids: torch.Tensor, status: torch.Tensor) -> int:
        st = int(status[0].item())
        err = row_error(st)
        if err is not None:
            raise err
        return int(ids[0].item()) & 0xFFFFFFFF

    def sample(self, logits: torch.Tensor, params: SamplingParams) -> int:
        """Sampler::sample (src/sampler.rs:32-35)."""
        return self.sample_logits(extract_logits(logits), params)

    def sample_logits(self, logits, params: SamplingParams) -> int:
        """Sampler::sample_logits (src/sampler.rs:44-54)."""
        row = self._row(logits)
        ids, status, _ = self._engine.sample(row, params, rng_states=self._state, want_probs=False)
        return self._result(ids, status)

    def sample_greedy(self, logits: torch.Tensor) -> int:
        """Sampler::sample_greedy (src/sampler.rs:63-66)."""
        return self.greedy_logits(extract_logits(logits))

    def greedy_logits(self, logits) -> int:
        """Sampler::greedy_logits (src/sampler.rs:75-88)."""
        row = self._row(logits)
        ids, status = self._engine.greedy(row)
        return self._result(ids, status)

    def sample_with_temp(self, logits: torch.Tensor, temperature: float) -> int:
        """Sampler::sample_with_temp (src/sampler.rs:97-105)."""
        row = extract_logits(logits).reshape(1, -1).to(self.device)
        ids, status, _ = self._engine.sample_with_temp(row, temperature, rng_states=self._state,
                                                       want_probs=False)
        return self._result(ids, status)

    def penalize(self, logits: torch.Tensor, tokens: Sequence[int], penalty: float) -> None:
        """Sampler::penalize (src/sampler.rs:107-109), in place on a device row."""
        row = logits.reshape(1, -1)
        toks = torch.tensor([int(t) & 0xFFFFFFFF for t in tokens], dtype=torch.int64)
        toks = toks.to(torch.int32) if toks.numel() == 0 else (toks - ((toks >> 31) << 32)).to(torch.int32)
        self._engine.penalize(row, toks, penalty)


def is_finite_float(x: float) -> bool:
    return not (math.isnan(x) or math.isinf(x))
