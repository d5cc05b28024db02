"""TEST INFRASTRUCTURE: build oracle/liboracle.so (the CPU restatement).

gcc -O2 -ffp-contract=off -fopenmp: every product and sum rounds as written,
OpenMP only splits independent rows. The reference itself is Python + MLX
(absent here) and has no C sources for these regions, so there is no
oracle/_ref build: nothing of the reference compiles on this machine.
"""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "mt_oracle.c"
LIB = HERE / "liboracle.so"
DEPS = [SRC, Path(__file__)]


def build_oracle(force: bool = False) -> Path:
    if not force and LIB.exists() and all(d.stat().st_mtime <= LIB.stat().st_mtime for d in DEPS):
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler for the oracle")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, "-O2", "-ffp-contract=off", "-fopenmp", "-shared", "-fPIC", "-Wall", "-Wno-unknown-pragmas",
           str(SRC), "-o", str(tmp), "-lm"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stderr}")
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build_oracle(force="--force" in sys.argv))
