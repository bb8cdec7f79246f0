"""Build recipe for the CPU oracle (test infrastructure): ``oracle/_build/liboracle.so``.

The oracle is a plain-C restatement of the reference's CPU backend; see
``marina_oracle.h``. Only the tests, ``__graft_entry__.smoke()`` and the benchmark's
CPU-baseline leg load it.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
SOURCES = [HERE / "marina_oracle.c"]
HEADERS = [HERE / "marina_oracle.h"]


def build(force: bool = False) -> Path:
    deps = SOURCES + HEADERS + [Path(__file__)]
    if not force and LIB.exists() and all(LIB.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return LIB
    LIB.parent.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = ["gcc", "-O3", "-std=c11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           *map(str, SOURCES), "-o", str(tmp), "-lm"]
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + proc.stdout)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
