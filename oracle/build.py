"""Build recipe for the oracle's C restatement (test infrastructure only).

Compiles oracle/oracle.c into oracle/_build/liboracle.so with gcc, OpenMP and
-ffp-contract=off (the restatement spells out every fused multiply-add).
The reference's own KNN kernel is built from its jt.code template by
oracle/build_ref.py (into oracle/_ref/).
"""

from __future__ import annotations

import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "oracle.c"
LIBRARY = HERE / "_build" / "liboracle.so"


def build(force: bool = False) -> Path:
    LIBRARY.parent.mkdir(exist_ok=True)
    if not force and LIBRARY.exists() and LIBRARY.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIBRARY
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-fno-fast-math", str(SOURCE), "-o", str(LIBRARY), "-lm"]
    subprocess.run(cmd, check=True)
    return LIBRARY


if __name__ == "__main__":
    print(build(force=True))
