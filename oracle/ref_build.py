"""Build the reference's own expert-path code as a CPU checker into oracle/_ref/ (TEST INFRASTRUCTURE).

Reads engine/mimo_stream/kernels.py of the reference tree WITHOUT importing it (it imports mlx, which
is absent here) and writes, into oracle/_ref/ (git-ignored; shipped to GPU boxes as a built artefact):
  * ref_header.inc, gateup_body.inc, down_body.inc - the Metal source strings HEADER, _GATEUP_SRC and
    _DOWN_SRC (kernels.py:19-123), compiled for the CPU by oracle/ref_kernels.cpp into libref_kernels.so;
  * group_routes_ref.py - the reference's pure-numpy group_routes (kernels.py:149-173).
Nothing from the reference is committed; this recipe regenerates everything from the read-only tree.
"""
from __future__ import annotations

import ast
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LIB = OUT / "libref_kernels.so"
ENV = "MIMO_REFERENCE_ROOT"  # the reference checkout (the directory holding engine/mimo_stream)


def reference_root() -> Path:
    root = os.environ.get(ENV)
    if not root:
        raise RuntimeError(f"set {ENV} to the reference checkout (the directory that holds engine/mimo_stream)")
    return Path(root)


def kernels_file() -> Path:
    return reference_root() / "engine" / "mimo_stream" / "kernels.py"


def extract():
    KERNELS = kernels_file()
    src = KERNELS.read_text()
    tree = ast.parse(src)
    strings, funcs = {}, {}
    for node in tree.body:
        if isinstance(node, ast.Assign) and len(node.targets) == 1 and isinstance(node.targets[0], ast.Name):
            if isinstance(node.value, ast.Constant) and isinstance(node.value.value, str):
                strings[node.targets[0].id] = node.value.value
        if isinstance(node, ast.FunctionDef):
            funcs[node.name] = ast.get_source_segment(src, node)
    for k in ("HEADER", "_GATEUP_SRC", "_DOWN_SRC"):
        if k not in strings:
            raise RuntimeError(f"{KERNELS}: {k} not found")
    if "group_routes" not in funcs:
        raise RuntimeError(f"{KERNELS}: group_routes not found")
    OUT.mkdir(exist_ok=True)
    (OUT / "ref_header.inc").write_text(strings["HEADER"])
    (OUT / "gateup_body.inc").write_text(strings["_GATEUP_SRC"])
    (OUT / "down_body.inc").write_text(strings["_DOWN_SRC"])
    (OUT / "group_routes_ref.py").write_text(
        f"# extracted at build time from {KERNELS} by oracle/ref_build.py; not committed\n"
        "import numpy as np\n\n\n" + funcs["group_routes"] + "\n")


def build(force: bool = False) -> Path:
    KERNELS = kernels_file()
    if not KERNELS.exists():
        if LIB.exists():
            return LIB
        raise RuntimeError(f"{ENV}={reference_root()}: {KERNELS.relative_to(reference_root())} not found")
    cpp = HERE / "ref_kernels.cpp"
    if not force and LIB.exists() and LIB.stat().st_mtime > max(cpp.stat().st_mtime, KERNELS.stat().st_mtime):
        return LIB
    extract()
    tmp = OUT / "libref_kernels.so.tmp"
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
           "-I", str(OUT), str(cpp), "-o", str(tmp)]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
