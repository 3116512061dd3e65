"""ctypes binding of the CPU oracle (oracle/sampling_ref.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, as the checker. The product never calls it.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np

from .build import LIB, build

RSO_OK = 0
RSO_NO_VALID_TOKENS = 1
RSO_VOCAB_OVERFLOW = 2


class RsoParams(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_k", ctypes.c_uint32),
        ("top_p", ctypes.c_float),
        ("repetition_penalty", ctypes.c_float),
        ("seed", ctypes.c_uint64),
    ]


class RsoResult(ctypes.Structure):
    _fields_ = [
        ("status", ctypes.c_int32),
        ("token", ctypes.c_uint32),
        ("consumed_draw", ctypes.c_int32),
        ("position", ctypes.c_uint32),
        ("prob", ctypes.c_float),
        ("n_survivors", ctypes.c_uint32),
        ("cdf_lo", ctypes.c_float),
        ("cdf_hi", ctypes.c_float),
    ]


RESULT_DTYPE = np.dtype([
    ("status", np.int32), ("token", np.uint32), ("consumed_draw", np.int32),
    ("position", np.uint32), ("prob", np.float32), ("n_survivors", np.uint32),
    ("cdf_lo", np.float32), ("cdf_hi", np.float32),
])
assert RESULT_DTYPE.itemsize == ctypes.sizeof(RsoResult)

_F = ctypes.POINTER(ctypes.c_float)
_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        P = ctypes.c_void_p
        SZ = ctypes.c_size_t
        sig = {
            "rso_sample_logits": (None, [P, SZ, ctypes.POINTER(RsoParams), ctypes.c_float, ctypes.POINTER(RsoResult)]),
            "rso_greedy_logits": (None, [P, SZ, ctypes.POINTER(RsoResult)]),
            "rso_sample_with_temp": (None, [P, SZ, ctypes.c_float, ctypes.c_float, ctypes.POINTER(RsoResult)]),
            "rso_pick": (None, [P, SZ, ctypes.POINTER(RsoParams), ctypes.c_float, ctypes.POINTER(RsoResult)]),
            "rso_filter": (SZ, [P, SZ, ctypes.POINTER(RsoParams), P, P]),
            "rso_topk_threshold": (ctypes.c_float, [P, SZ, ctypes.c_float, ctypes.c_uint32]),
            "rso_topp_edge": (SZ, [P, SZ, ctypes.POINTER(RsoParams), _F, _F]),
            "rso_softmax": (None, [P, SZ, P]),
            "rso_argmax": (SZ, [P, SZ]),
            "rso_apply_repetition_penalty": (None, [P, SZ, P, SZ, ctypes.c_float]),
            "rso_sample_rows": (None, [P, SZ, SZ, SZ, ctypes.POINTER(RsoParams), P, P, ctypes.c_int]),
            "rso_greedy_rows": (None, [P, SZ, SZ, SZ, P, ctypes.c_int]),
            "rso_sample_with_temp_rows": (None, [P, SZ, SZ, SZ, ctypes.c_float, P, P, ctypes.c_int]),
            "rso_rng_next_u64": (ctypes.c_uint64, [ctypes.POINTER(ctypes.c_uint64)]),
            "rso_rng_f32": (ctypes.c_float, [ctypes.POINTER(ctypes.c_uint64)]),
            "rso_expf_many": (None, [P, SZ, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def params(temperature: float, top_k: int, top_p: float, repetition_penalty: float = 1.0,
           seed: int = 0) -> RsoParams:
    return RsoParams(temperature, top_k & 0xFFFFFFFF, top_p, repetition_penalty,
                     seed & 0xFFFFFFFFFFFFFFFF)


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


@dataclass
class Result:
    status: int
    token: int
    consumed_draw: bool
    position: int
    prob: float
    n_survivors: int
    cdf_lo: float
    cdf_hi: float


def _res(r: RsoResult) -> Result:
    return Result(r.status, r.token, bool(r.consumed_draw), r.position, r.prob, r.n_survivors,
                  r.cdf_lo, r.cdf_hi)


def sample_logits(logits, p: RsoParams, u: float = 0.0) -> Result:
    x = _f32(logits)
    r = RsoResult()
    lib().rso_sample_logits(x.ctypes.data, x.size, ctypes.byref(p), ctypes.c_float(u), ctypes.byref(r))
    return _res(r)


def greedy_logits(logits) -> Result:
    x = _f32(logits)
    r = RsoResult()
    lib().rso_greedy_logits(x.ctypes.data, x.size, ctypes.byref(r))
    return _res(r)


def sample_with_temp(logits, temperature: float, u: float = 0.0) -> Result:
    x = _f32(logits)
    r = RsoResult()
    lib().rso_sample_with_temp(x.ctypes.data, x.size, ctypes.c_float(temperature), ctypes.c_float(u),
                               ctypes.byref(r))
    return _res(r)


def pick(logits, p: RsoParams, u: float = 0.0) -> Result:
    x = _f32(logits)
    r = RsoResult()
    lib().rso_pick(x.ctypes.data, x.size, ctypes.byref(p), ctypes.c_float(u), ctypes.byref(r))
    return _res(r)


def filter_(logits, p: RsoParams) -> tuple[np.ndarray, np.ndarray]:
    x = _f32(logits)
    idx = np.empty(max(1, x.size), dtype=np.uint32)
    val = np.empty(max(1, x.size), dtype=np.float32)
    n = lib().rso_filter(x.ctypes.data, x.size, ctypes.byref(p), idx.ctypes.data, val.ctypes.data)
    return idx[:n].copy(), val[:n].copy()


def topp_edge(logits, p: RsoParams) -> tuple[int, float, float]:
    """(kept count, running sum before, running sum after) at the top-p cut."""
    x = _f32(logits)
    b, a = ctypes.c_float(), ctypes.c_float()
    n = lib().rso_topp_edge(x.ctypes.data, x.size, ctypes.byref(p), ctypes.byref(b), ctypes.byref(a))
    return int(n), float(b.value), float(a.value)


def topk_threshold(logits, temperature: float, k: int) -> float:
    x = _f32(logits)
    return float(lib().rso_topk_threshold(x.ctypes.data, x.size, ctypes.c_float(temperature), k))


def softmax(values) -> np.ndarray:
    x = _f32(values)
    out = np.empty(max(1, x.size), dtype=np.float32)
    lib().rso_softmax(x.ctypes.data, x.size, out.ctypes.data)
    return out[:x.size].copy()


def argmax(values) -> Optional[int]:
    x = _f32(values)
    r = lib().rso_argmax(x.ctypes.data, x.size)
    return None if r == ctypes.c_size_t(-1).value else int(r)


def apply_repetition_penalty(logits, tokens, penalty: float) -> np.ndarray:
    x = _f32(logits).copy()
    t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
    lib().rso_apply_repetition_penalty(x.ctypes.data, x.size, t.ctypes.data, t.size,
                                       ctypes.c_float(penalty))
    return x


def sample_rows(logits: np.ndarray, p: RsoParams, u: Optional[np.ndarray], threads: int = 1) -> np.ndarray:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    rows, n = x.shape
    out = np.zeros(rows, dtype=RESULT_DTYPE)
    uu = None if u is None else np.ascontiguousarray(u, dtype=np.float32)
    lib().rso_sample_rows(x.ctypes.data, rows, n, n, ctypes.byref(p),
                          None if uu is None else uu.ctypes.data, out.ctypes.data, threads)
    return out


def greedy_rows(logits: np.ndarray, threads: int = 1) -> np.ndarray:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    rows, n = x.shape
    out = np.zeros(rows, dtype=RESULT_DTYPE)
    lib().rso_greedy_rows(x.ctypes.data, rows, n, n, out.ctypes.data, threads)
    return out


def sample_with_temp_rows(logits: np.ndarray, temperature: float, u: Optional[np.ndarray],
                          threads: int = 1) -> np.ndarray:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    rows, n = x.shape
    out = np.zeros(rows, dtype=RESULT_DTYPE)
    uu = None if u is None else np.ascontiguousarray(u, dtype=np.float32)
    lib().rso_sample_with_temp_rows(x.ctypes.data, rows, n, n, ctypes.c_float(temperature),
                                    None if uu is None else uu.ctypes.data, out.ctypes.data, threads)
    return out


def rng_stream(seed: int, count: int) -> np.ndarray:
    """`count` successive uniforms of the wyrand restatement from `seed`."""
    st = ctypes.c_uint64(seed & 0xFFFFFFFFFFFFFFFF)
    return np.array([lib().rso_rng_f32(ctypes.byref(st)) for _ in range(count)], dtype=np.float32)


def expf(x) -> np.ndarray:
    a = _f32(x)
    out = np.empty_like(a)
    lib().rso_expf_many(a.ctypes.data, a.size, out.ctypes.data)
    return out
