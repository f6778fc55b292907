"""Build the sm_100a shared library in-tree: mimo_moe/libmimo_moe.so (nvcc, no torch extension)."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parent.parent / "include"
LIB = PKG / "libmimo_moe.so"
SOURCES = ["api.cu", "router.cu", "dispatch.cu", "experts.cu", "synth.cu", "noalloc.cu", "tma.cu", "tc_experts.cu", "peer.cu", "norm.cu", "ep_plan.cu", "loader.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    return "nvcc"


def sources():
    return [CSRC / s for s in SOURCES]


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "mimo_moe.h"]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every .cu for sm_100a (-lineinfo, -O3) and link libmimo_moe.so next to this file."""
    if not force and not _stale():
        return LIB
    build_dir = PKG.parent / "_build"
    build_dir.mkdir(exist_ok=True)
    common = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-I", str(INCLUDE), "--expt-relaxed-constexpr"]
    if ptxas_verbose:
        common += ["-Xptxas", "-v"]
    objs, procs = [], []
    for src in sources():
        obj = build_dir / (src.stem + ".o")
        objs.append(obj)
        cmd = common + ["-c", str(src), "-o", str(obj)]
        procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    ok = True
    for cmd, pr in procs:
        out, _ = pr.communicate()
        if verbose or pr.returncode != 0:
            sys.stderr.write(out)
        if pr.returncode != 0:
            ok = False
            sys.stderr.write(f"\nFAILED: {' '.join(cmd)}\n")
    if not ok:
        raise RuntimeError("nvcc failed")
    tmp = LIB.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp)] + [str(o) for o in objs] + ["-lpthread"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_verbose="-v" in sys.argv)
    print(LIB)
