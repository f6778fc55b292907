"""Build oracle/cpu_mxfp4.c into oracle/libmimo_cpu_port.so (TEST INFRASTRUCTURE: the native form of the timed CPU
baseline; git-ignored as a built file, shipped to GPU boxes with the tree).

    python oracle/cpu_port_build.py [--force]
"""
from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "cpu_mxfp4.c"
LIB = HERE / "libmimo_cpu_port.so"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= max(SRC.stat().st_mtime, Path(__file__).stat().st_mtime):
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler for the CPU baseline")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([cc, "-O3", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-o", str(tmp), str(SRC), "-lm"],
                   check=True)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
