"""Build the sm_100a shared libraries in-tree (nvcc, no torch extension): mimo_moe/libmimo_moe.so (the
MoE block, include/mimo_moe.h) and mimo_moe/libmimo_moe_testkit.so (synthetic pools and the tensor-peak
probe for tests and benchmarks, include/mimo_moe_testkit.h)."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parent.parent / "include"
LIB = PKG / "libmimo_moe.so"
LIB_TESTKIT = PKG / "libmimo_moe_testkit.so"
SOURCES = ["api.cu", "router.cu", "dispatch.cu", "experts.cu", "noalloc.cu", "tma.cu", "tc_experts.cu", "peer.cu",
           "norm.cu", "ep_plan.cu", "layer.cu", "attn_tc.cu", "linear.cu", "loader.cpp", "slot_cache.cpp"]
TESTKIT_SOURCES = ["synth.cu", "testkit.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    return "nvcc"


def sources():
    return [CSRC / s for s in SOURCES + TESTKIT_SOURCES]


def _stale() -> bool:
    if not LIB.exists() or not LIB_TESTKIT.exists():
        return True
    t = min(LIB.stat().st_mtime, LIB_TESTKIT.stat().st_mtime)
    deps = sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every .cu for sm_100a (-lineinfo, -O3) and link both libraries next to this file."""
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
    for lib, names in ((LIB, SOURCES), (LIB_TESTKIT, TESTKIT_SOURCES)):
        tmp = lib.with_suffix(".so.tmp")
        mine = [str(build_dir / (Path(n).stem + ".o")) for n in names]
        subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp)] + mine + ["-lpthread"], check=True)
        os.replace(tmp, lib)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_verbose="-v" in sys.argv)
    print(LIB)
