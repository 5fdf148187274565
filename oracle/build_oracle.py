"""Compile the C restatement of the oracle (test infrastructure) into oracle/libasu_oracle.so.

    python -m oracle.build_oracle

The reference's own kernels are AscendC / AICPU code that needs the CANN toolchain, so
no part of the reference path is compiled here; this builds only the restatement.
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "asu_oracle.c"
LIB = HERE / "libasu_oracle.so"


def build() -> Path:
    if LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler found for the oracle")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([cc, "-O2", "-std=c11", "-fPIC", "-shared", "-pthread", str(SRC), "-o", str(tmp)], check=True)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build())
