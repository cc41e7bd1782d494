"""Builds the oracle's C restatement into ``oracle/_build/libjc_oracle.so`` (test infrastructure).

Compiled with ``-ffp-contract=off`` and without fast-math so that double sums and products round
as Java's do. The reference itself (Java 22, TornadoVM) cannot be built here: there is no JDK, so
no ``oracle/_ref`` is produced.
"""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build" / "libjc_oracle.so"
FLAGS = ["-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math", "-pthread"]


def build(verbose: bool = False) -> Path:
    sources = sorted(HERE.glob("*.c"))
    headers = sorted(HERE.glob("*.h"))
    if OUT.exists() and all(p.stat().st_mtime <= OUT.stat().st_mtime for p in sources + headers):
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    cmd = ["gcc", *FLAGS, "-o", str(OUT), *map(str, sources), "-lm"]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
