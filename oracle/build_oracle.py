"""Build recipe for the oracle's C restatement (test infrastructure only).

    python oracle/build_oracle.py

compiles oracle/decode_ref.c with gcc and OpenMP into
oracle/liboracle_decode.so. __graft_entry__.build() runs the same recipe.
"""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
SOURCE = ORACLE_DIR / "decode_ref.c"
LIB = ORACLE_DIR / "liboracle_decode.so"


def build_c_oracle(force: bool = False) -> Path:
    """Compile decode_ref.c (when the source is newer than the library)."""
    if not force and LIB.exists() and LIB.stat().st_mtime >= SOURCE.stat().st_mtime:
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler (gcc) for the oracle's C restatement")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, "-O3", "-fopenmp", "-fPIC", "-shared", str(SOURCE), "-o", str(tmp), "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle C build failed:\n{r.stdout}\n{r.stderr}")
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build_c_oracle(force="--force" in sys.argv))
