"""The C-ABI library loads and exports every symbol include/*.h declares (CPU only:
no call here touches a GPU)."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from rusticide_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        for m in re.finditer(r"RSC_API\s+[^;(]*?\b(rsc_\w+)\s*\(", h.read_text()):
            names.add(m.group(1))
    return names


def test_header_declares_the_abi():
    names = declared_symbols()
    for must in ["rsc_sampler_create", "rsc_sampler_destroy", "rsc_sample", "rsc_sample_ex",
                 "rsc_greedy", "rsc_sample_with_temp", "rsc_pick", "rsc_pick_host",
                 "rsc_penalize", "rsc_rng_seed", "rsc_shard_partial", "rsc_shard_merge",
                 "rsc_shard_record_bytes", "rsc_expf", "rsc_launch_count", "rsc_status_string",
                 "rsc_debug_hold_scratch",
                 "rsc_abi_version"]:
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    missing = declared_symbols() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    for name in declared_symbols():
        assert hasattr(lib, name)
        assert name in _lib.SIGNATURES, f"no ctypes signature for {name}"


def test_compute_free_calls():
    lib = _lib.load()
    assert lib.rsc_abi_version() == 2
    assert lib.rsc_status_string(_lib.RSC_OK) == b"ok"
    assert lib.rsc_status_string(_lib.RSC_ERR_INVALID_SHAPE) == b"invalid shape"
    assert lib.rsc_shard_record_bytes(40) == 32 + 8 * (40 + _lib.RSC_SHARD_TIE_CAP)
    assert lib.rsc_shard_record_bytes(41) % 16 == 0
    assert ctypes.sizeof(_lib.RscParams) == 24
    # Null handles are rejected before any device work.
    assert lib.rsc_sample(None, None, 0, 0, 0, None, None, None, None, None, None, None) == \
        _lib.RSC_ERR_NOT_INITIALIZED
    assert lib.rsc_launch_count(None) == 0


def test_header_compiles_as_c():
    src = '#include "rusticide_cuda.h"\nint main(void){ rsc_params p = {0}; (void)p; return 0; }\n'
    res = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"), "-x", "c",
                          "-", "-o", "/dev/null"], input=src, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


def test_rust_binding_declares_every_symbol():
    """rust/rusticide-cuda/src/ffi.rs is the binding a Rust caller links (it is
    not compiled here: no Rust toolchain on this image), so its extern block is
    checked as text against the header."""
    ffi = (ROOT / "rust" / "rusticide-cuda" / "src" / "ffi.rs").read_text()
    bound = set(re.findall(r"\bfn\s+(rsc_\w+)\s*\(", ffi))
    missing = declared_symbols() - bound
    assert not missing, f"declared in the header but not bound in ffi.rs: {sorted(missing)}"
    extra = bound - declared_symbols()
    assert not extra, f"bound in ffi.rs but not declared in the header: {sorted(extra)}"


def header_parameter_counts() -> dict[str, int]:
    header = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "rusticide_cuda.h").read_text(), flags=re.S)
    want = {}
    for m in re.finditer(r"RSC_API\s+[^;(]*?\b(rsc_\w+)\s*\(([^;]*?)\)\s*;", header, flags=re.S):
        args = m.group(2).strip()
        want[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return want


def test_ctypes_signatures_match_the_header():
    want = header_parameter_counts()
    assert want, "no declarations parsed from the header"
    mismatched = {k: (n, len(_lib.SIGNATURES[k][1])) for k, n in want.items()
                  if len(_lib.SIGNATURES[k][1]) != n}
    assert not mismatched, f"(header, ctypes) parameter counts differ: {mismatched}"


def test_rust_binding_parameter_counts_match_the_header():
    want = header_parameter_counts()
    ffi = (ROOT / "rust" / "rusticide-cuda" / "src" / "ffi.rs").read_text()
    got = {}
    for m in re.finditer(r"\bfn\s+(rsc_\w+)\s*\(([^)]*)\)", ffi, flags=re.S):
        args = m.group(2).strip().rstrip(",")
        got[m.group(1)] = 0 if not args else args.count(",") + 1
    assert want, "no declarations parsed from the header"
    mismatched = {k: (want[k], got.get(k)) for k in want if want[k] != got.get(k)}
    assert not mismatched, f"(header, ffi.rs) parameter counts differ: {mismatched}"
