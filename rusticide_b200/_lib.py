"""ctypes binding of librusticide_cuda.so (the C ABI in include/rusticide_cuda.h).

The library is the product path: there is no fallback. If the shared object is
missing this module raises at import time, naming the build command.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "librusticide_cuda.so"

# Call-level statuses (rsc_status).
RSC_OK = 0
RSC_ERR_INVALID_ARGUMENT = 1
RSC_ERR_INVALID_SHAPE = 2
RSC_ERR_VOCAB_TOO_LARGE = 3
RSC_ERR_CAPACITY = 4
RSC_ERR_CUDA = 5
RSC_ERR_NOT_INITIALIZED = 6
RSC_ERR_NO_DEVICE = 7

# Per-row statuses (low byte) and flags.
RSC_ROW_OK = 0
RSC_ROW_NO_VALID_TOKENS = 1
RSC_ROW_VOCAB_OVERFLOW = 2
RSC_ROW_INTERNAL = 3
RSC_ROW_FLAG_DRAW_NEAR_BOUNDARY = 1 << 8
RSC_ROW_FLAG_LARGE_PATH = 1 << 9

RSC_SHARD_TIE_CAP = 24
RSC_NOALLOC_SCRATCH_BYTES = 64 << 20
RSC_NOALLOC_MAX_VOCAB = RSC_NOALLOC_SCRATCH_BYTES // 16


class RscParams(ctypes.Structure):
    """rsc_params == SamplingParams, crates/rusticide-sampling/src/params.rs:5-12."""

    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_k", ctypes.c_uint32),
        ("top_p", ctypes.c_float),
        ("repetition_penalty", ctypes.c_float),
        ("seed", ctypes.c_uint64),
    ]


class RscPeerExchange(ctypes.Structure):
    """rsc_peer_exchange: device addresses of the arrays the ranks share."""

    _fields_ = [
        ("d_peer_records", ctypes.c_void_p),
        ("d_ready_records", ctypes.c_void_p),
        ("d_ready_results_ptrs", ctypes.c_void_p),
        ("d_done_counter", ctypes.c_void_p),
        ("d_peer_ids", ctypes.c_void_p),
        ("d_peer_status", ctypes.c_void_p),
        ("d_peer_probs", ctypes.c_void_p),
    ]


class RscSampleExtras(ctypes.Structure):
    """rsc_sample_extras."""

    _fields_ = [
        ("d_n_survivors", ctypes.c_void_p),
        ("d_survivor_ids", ctypes.c_void_p),
        ("survivor_cap", ctypes.c_size_t),
        ("d_survivor_probs", ctypes.c_void_p),
        ("d_row_logsumexp", ctypes.c_void_p),
        ("d_token_logprob", ctypes.c_void_p),
        ("d_survivor_logprobs", ctypes.c_void_p),
    ]


# Every symbol the header declares, with its ctypes signature.
_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_ST = ctypes.c_int
SIGNATURES = {
    "rsc_status_string": (ctypes.c_char_p, [_ST]),
    "rsc_abi_version": (ctypes.c_int, []),
    "rsc_sampler_create": (_ST, [ctypes.c_int, _SZ, _SZ, ctypes.POINTER(_P)]),
    "rsc_sampler_destroy": (_ST, [_P]),
    "rsc_sample": (_ST, [_P, _P, _SZ, _SZ, _SZ, ctypes.POINTER(RscParams), _P, _P, _P, _P, _P, _P]),
    "rsc_sample_rows": (_ST, [_P, _P, _SZ, _SZ, _SZ, ctypes.POINTER(RscParams), _P, _P, _P, _P, _P,
                             _P]),
    "rsc_sample_ex": (_ST, [_P, _P, _SZ, _SZ, _SZ, ctypes.POINTER(RscParams), _P, _P, _P, _P, _P,
                            _P, _P]),
    "rsc_greedy": (_ST, [_P, _P, _SZ, _SZ, _SZ, _P, _P, _P]),
    "rsc_sample_with_temp": (_ST, [_P, _P, _SZ, _SZ, _SZ, ctypes.c_float, _P, _P, _P, _P, _P, _P]),
    "rsc_pick": (_ST, [_P, _P, _SZ, _SZ, _SZ, ctypes.POINTER(RscParams), _P, _P, _P, _P, _P, _P]),
    "rsc_pick_host": (_ST, [_P, _P, _SZ, _SZ, ctypes.POINTER(RscParams), _P, _P, _P, _P]),
    "rsc_penalize": (_ST, [_P, _P, _SZ, _SZ, _SZ, _P, _SZ, ctypes.c_float, _P]),
    "rsc_rng_seed": (_ST, [_P, _P, _SZ, _P]),
    "rsc_shard_record_bytes": (_SZ, [ctypes.c_uint32]),
    "rsc_shard_partial": (_ST, [_P, _P, _SZ, _SZ, _SZ, _SZ, _SZ, ctypes.POINTER(RscParams), _P, _P]),
    "rsc_shard_merge": (_ST, [_P, _P, _SZ, _SZ, _SZ, ctypes.POINTER(RscParams), _P, _P, _P, _P, _P, _P]),
    "rsc_shard_merge_peers": (_ST, [_P, ctypes.POINTER(RscPeerExchange), ctypes.c_uint32, _SZ, _SZ,
                                    _SZ, _SZ, ctypes.POINTER(RscParams), _P, _P, _P]),
    "rsc_shard_collect": (_ST, [_P, ctypes.c_uint32, _SZ, _SZ, _P, _P, _P, _P, _P, _P, _P]),
    "rsc_shard_publish": (_ST, [_P, _SZ, _SZ, ctypes.c_uint32, _P]),
    "rsc_sample_noalloc": (_ST, [_P, _SZ, _SZ, _SZ, ctypes.POINTER(RscParams), _P, _P, _P, _P, _P,
                                 _P]),
    "rsc_lmhead_logits": (_ST, [_P, _P, _P, _SZ, _SZ, _SZ, _P, _P]),
    "rsc_lmhead_partial": (_ST, [_P, _P, _P, _SZ, _SZ, _SZ, _SZ, _SZ, ctypes.POINTER(RscParams),
                                 _P, _P]),
    "rsc_lmhead_sample": (_ST, [_P, _P, _P, _SZ, _SZ, _SZ, ctypes.POINTER(RscParams), _P, _P, _P,
                                _P, _P, _P]),
    "rsc_expf": (_ST, [_P, _P, _SZ, _P]),
    "rsc_launch_count": (ctypes.c_uint64, [_P]),
    "rsc_debug_hold_scratch": (_ST, [_P, ctypes.c_int, _P]),
}


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(
            f"{p} is missing: build the CUDA library first "
            "(python -c 'import __graft_entry__ as g; g.build()' or python rusticide_b200/build.py)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = load()
    return _LIB


def status_string(code: int) -> str:
    return lib().rsc_status_string(code).decode()


class RscError(RuntimeError):
    """A call-level error of the C ABI."""

    def __init__(self, code: int, what: str):
        super().__init__(f"{what}: {status_string(code)} ({code})")
        self.code = code


def check(code: int, what: str) -> None:
    if code != RSC_OK:
        raise RscError(code, what)
