"""Build recipe for the C half of the CPU oracle (test infrastructure only).

Compiles ``oracle/dyn_int8.c`` with gcc into ``oracle/liboracle.so``.  The
flags keep IEEE fp32 semantics: no fast-math and no implicit contraction of
``a * b + c`` into a fused multiply-add (the one fused operation the restated
algorithm needs is spelled ``fmaf`` in the source).
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "dyn_int8.c"
LIB = HERE / "liboracle.so"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    tmp = LIB.with_suffix(".so.tmp%d" % os.getpid())
    cmd = ["gcc", "-O3", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off", "-fno-fast-math",
           "-o", str(tmp), str(SRC), "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
