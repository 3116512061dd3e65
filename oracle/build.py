"""Build recipe of the CPU oracle liboracle_sampling.so (test infrastructure).

g++ without fast-math and with -ffp-contract=off, so that every binary32
operation of the restatement is one IEEE operation, as in the Rust reference.
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "sampling_ref.cpp"
LIB = HERE / "liboracle_sampling.so"
FLAGS = ["-O2", "-std=c++17", "-fno-fast-math", "-ffp-contract=off", "-fPIC", "-shared",
         "-pthread"]


def build(force: bool = False) -> Path:
    deps = [SRC, HERE / "sampling_ref.h"]
    if not force and LIB.exists() and all(d.stat().st_mtime <= LIB.stat().st_mtime for d in deps):
        return LIB
    cmd = ["g++", *FLAGS, str(SRC), "-o", str(LIB), "-lm"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("oracle build failed")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
