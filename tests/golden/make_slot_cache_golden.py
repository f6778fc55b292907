"""Record runs of the reference's own expert slot table (engine/mimo_stream/cache.py, SlotCache) as golden
fixtures: tests/golden/slot_cache.json.

    MIMO_REFERENCE_ROOT=<reference checkout> python tests/golden/make_slot_cache_golden.py

cache.py imports only numpy, so its class runs here unchanged (loaded by path; nothing of it is copied).  Each
run is a seeded sequence of the engine's calls (model.py:160-167 preload, 191 resolve of a decode step's
distinct experts, 327 resolve of predicted experts with count=False, stats=False, 353 decay every 16 decode
tokens), with skewed, drifting expert popularity; every step records the call, its arguments, the loads it
returned and the hit / miss counters after it."""
import importlib.util
import json
import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().with_name("slot_cache.json")


# (seed, slots, experts, decode steps, preload, most tokens per step)
RUNS = [(1, 64, 256, 240, True, 1),      # decode B=1, a quarter of the experts resident
        (2, 96, 256, 160, True, 4),      # small verify batches
        (3, 48, 256, 120, False, 2),     # starting empty: ties among empty slots
        (4, 16, 64, 200, True, 1)]       # a small table: many evictions


def reference_slot_cache(root=None):
    root = root or os.environ.get("MIMO_REFERENCE_ROOT")
    if not root:
        sys.exit("set MIMO_REFERENCE_ROOT to the reference checkout (the directory holding engine/mimo_stream)")
    path = Path(root) / "engine" / "mimo_stream" / "cache.py"
    spec = importlib.util.spec_from_file_location("reference_slot_cache", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.SlotCache


def _run(SlotCache, seed: int, S: int, E: int, steps: int, preload: bool, max_tokens: int):
    rng = np.random.default_rng(seed)
    c = SlotCache(S, E)
    log = []
    if preload:
        order = [int(e) for e in rng.permutation(E)[:S]]
        loads = c.preload(order)
        log.append({"op": "preload", "experts": order, "loads": [[int(e), int(s)] for e, s in loads],
                    "hits": int(c.hits), "misses": int(c.misses)})
    # popularity: a Zipf-like base over a random permutation, drifting by re-permuting a few ranks per step
    rank = rng.permutation(E)
    base = 1.0 / np.arange(1, E + 1) ** 1.1
    for step in range(steps):
        if step % 7 == 0:
            i, j = rng.integers(0, E, 2)
            rank[[i, j]] = rank[[j, i]]
        p = np.empty(E)
        p[rank] = base
        p /= p.sum()
        T = int(rng.integers(1, max_tokens + 1))
        routes = np.stack([rng.choice(E, 8, replace=False, p=p) for _ in range(T)])
        needed = np.unique(routes)
        loads = c.resolve(needed)
        log.append({"op": "resolve", "needed": [int(e) for e in needed], "count": True, "stats": True,
                    "loads": [[int(e), int(s)] for e, s in loads], "hits": int(c.hits), "misses": int(c.misses)})
        if step % 5 == 4:   # a predicted next-layer set, loaded without counting (model.py:327)
            pred = np.unique(rng.choice(E, 8, replace=False, p=p))
            loads = c.resolve(pred, count=False, stats=False)
            log.append({"op": "resolve", "needed": [int(e) for e in pred], "count": False, "stats": False,
                        "loads": [[int(e), int(s)] for e, s in loads], "hits": int(c.hits), "misses": int(c.misses)})
        if step % 16 == 15:
            c.decay()
            log.append({"op": "decay"})
    return {"seed": seed, "S": S, "E": E, "preload": preload, "log": log}


def runs(SlotCache):
    return [_run(SlotCache, *r) for r in RUNS]


def main():
    OUT.write_text(json.dumps({"source": "engine/mimo_stream/cache.py (SlotCache), run unchanged",
                               "runs": runs(reference_slot_cache())}, separators=(",", ":")))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
