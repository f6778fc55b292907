"""Generate the golden fixtures of this directory from the reference's own code (run in a container that
has the read-only reference tree; the outputs are committed, the reference code is not).

  MIMO_REFERENCE_ROOT=<reference checkout> python oracle/ref_build.py && python tests/golden/make_golden.py

Sources of truth:
  * group_routes.npz - the reference's numpy group_routes (engine/mimo_stream/kernels.py:149-173),
    extracted verbatim by oracle/ref_build.py and executed here;
  * kernels_small.npz / kernels_full.npz - the reference's Metal kernels A/B (kernels.py:33-123)
    compiled for the CPU by oracle/ref_build.py + oracle/ref_kernels.cpp, driven by the reference's
    group_routes, followed by the gather + fixed-order sum of kernels.py:198-199.
Expert pools come from the seeded generator in oracle/synth.py (the fixtures store its seed and
shapes, not the pool bytes); the bf16 sigmoid table handed to the kernels is oracle.sigmoid_table_bits().
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import mimo_oracle as O  # noqa: E402
from oracle import ref_runner as RR  # noqa: E402
from oracle import synth  # noqa: E402

OUT = Path(__file__).resolve().parent


def group_routes_cases():
    rng = np.random.default_rng(1234)
    cases = []
    for M in (1, 2, 3, 4, 8):
        inds = np.stack([rng.choice(256, 8, replace=False) for _ in range(M)])
        if M > 1:
            inds[1, :4] = inds[0, :4]
        cases.append((inds, rng.random((M, 8)).astype(np.float32), 8))
    cases.append((np.tile(np.arange(4), (8, 1)), np.full((8, 4), 0.25, np.float32), 8))   # R saturated
    cases.append((np.array([[5, 5, 9, 1], [9, 9, 9, 2]]), rng.random((2, 4)).astype(np.float32), 8))  # repeats
    cases.append((rng.integers(0, 24, size=(6, 8)), rng.random((6, 8)).astype(np.float32), 16))
    out = {}
    for i, (inds, sc, R) in enumerate(cases):
        uids, urows, ucnt, uw, gidx = RR.group_routes(inds, sc, R)
        out.update({f"c{i}_inds": inds.astype(np.int32), f"c{i}_scores": sc, f"c{i}_R": np.int32(R),
                    f"c{i}_uids": uids.astype(np.int32), f"c{i}_urows": urows, f"c{i}_ucnt": ucnt,
                    f"c{i}_uw": uw, f"c{i}_gidx": gidx})
    try:        # the overflow rule (kernels.py:167-168)
        RR.group_routes(np.zeros((3, 1), np.int64), np.ones((3, 1), np.float32), 2)
        raised = 0
    except ValueError:
        raised = 1
    out["overflow_raises"] = np.int32(raised)
    out["ncases"] = np.int32(len(cases))
    np.savez_compressed(OUT / "group_routes.npz", **out)


def kernel_cases(name, H, I, S, Ms, seed, layer, k):
    shapes = {"gate": (I, H), "up": (I, H), "down": (H, I)}
    sp = synth.SynthPool(seed, layer, shapes)
    pool = {f"{n}_{kk}": np.stack([sp[f"{n}_{kk}"][e] for e in range(S)]) for n in shapes for kk in "ws"}
    rng = np.random.default_rng(seed + 77)
    out = {"H": np.int32(H), "I": np.int32(I), "S": np.int32(S), "seed": np.int32(seed),
           "layer": np.int32(layer), "Ms": np.array(Ms, np.int32)}
    sig = O.sigmoid_table_bits()
    for M in Ms:
        x = O.f32_to_bf16_bits(rng.standard_normal((M, H)).astype(np.float32))
        inds = np.stack([rng.choice(S, k, replace=False) for _ in range(M)])
        if M > 1:
            inds[1, :k // 2] = inds[0, :k // 2]
        sc = rng.random((M, k)).astype(np.float32)
        sc /= sc.sum(1, keepdims=True)
        uids, urows, ucnt, uw, gidx = RR.group_routes(inds, sc)
        y, h, part = RR.moe_experts(x, pool, uids.astype(np.int32), urows, ucnt, uw, gidx, sig)
        out.update({f"M{M}_x": x, f"M{M}_inds": inds.astype(np.int32), f"M{M}_scores": sc, f"M{M}_y": y,
                    f"M{M}_part_sum": part.astype(np.float64).sum(axis=2)})
        if H * I <= 512 * 256:
            out[f"M{M}_h"] = h
    np.savez_compressed(OUT / name, **out)


if __name__ == "__main__":
    if not RR.available():
        sys.exit("build oracle/_ref first: python oracle/ref_build.py")
    group_routes_cases()
    kernel_cases("kernels_small.npz", 512, 256, 6, [1, 2, 4, 8], seed=5, layer=0, k=4)
    kernel_cases("kernels_full.npz", 4096, 2048, 12, [1, 2, 8], seed=0, layer=0, k=8)
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)
