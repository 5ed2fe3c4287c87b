"""Build recipe of the CPU oracle (test infrastructure): oracle/_build/libsrs_oracle.so.

    python oracle/build_oracle.py [--force]

-ffp-contract=off keeps every FP32 operation separately rounded; the only
fused multiply-adds are the explicit fmaf() calls that mirror PyTorch's CPU
kernels.  No -ffast-math, no x87 (x86-64 SSE arithmetic).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "srs_oracle.c"
LIBRARY = HERE / "_build" / "libsrs_oracle.so"
FLAGS = ["-O2", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off", "-fno-fast-math"]


def build(force: bool = False) -> Path:
    if not force and LIBRARY.exists() and LIBRARY.stat().st_mtime >= max(
        SOURCE.stat().st_mtime, Path(__file__).stat().st_mtime
    ):
        return LIBRARY
    cc = os.environ.get("CC") or shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("a C compiler (gcc) is required to build the oracle")
    LIBRARY.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIBRARY.with_suffix(".so.tmp")
    subprocess.run([cc, *FLAGS, str(SOURCE), "-o", str(tmp), "-lm"], check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
