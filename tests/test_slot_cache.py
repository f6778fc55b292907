"""The expert residency table (engine/mimo_stream/cache.py:13-65) on the CPU: the oracle's restatement pinned to
recorded runs of the reference's own class (tests/golden/slot_cache.json, made by
tests/golden/make_slot_cache_golden.py), and the library's native table (mimo_moe_slot_cache_*, behind
mimo_moe.SlotCache) equal to the oracle step for step on seeded call sequences."""
import copy
import json
from pathlib import Path

import numpy as np
import pytest

from oracle.slot_cache import SlotCache as OracleSlotCache

GOLDEN = Path(__file__).resolve().parent / "golden" / "slot_cache.json"


def _runs():
    return json.loads(GOLDEN.read_text())["runs"]


@pytest.mark.parametrize("run", range(4))
def test_oracle_matches_the_reference_runs(run):
    """Same missing experts in the same order, same hit / miss counters after every call, and victims of
    equal scores (the reference's np.argpartition may take another slot among equal scores, so the run
    continues with the reference's own choice)."""
    r = _runs()[run]
    c = OracleSlotCache(r["S"], r["E"])
    other_choice = 0
    for entry in r["log"]:
        if entry["op"] == "preload":
            assert [list(x) for x in c.preload(entry["experts"])] == entry["loads"]
        elif entry["op"] == "decay":
            c.decay()
            continue
        else:
            ref = [tuple(x) for x in entry["loads"]]
            mine_c = copy.deepcopy(c)
            mine = mine_c.resolve(entry["needed"], entry["count"], entry["stats"])
            assert [e for e, _ in mine] == [e for e, _ in ref]
            if ref:
                assert sorted(mine_c.scores[[s for _, s in mine]]) == sorted(mine_c.scores[[s for _, s in ref]])
                other_choice += sorted(s for _, s in mine) != sorted(s for _, s in ref)
            c.resolve(entry["needed"], entry["count"], entry["stats"], victims=[s for _, s in ref])
        assert (c.hits, c.misses) == (entry["hits"], entry["misses"])
    # the ties exist (run 2 starts empty: every empty slot scores -1)
    if run == 2:
        assert other_choice > 0


def _sequence(seed, S, E, steps, preload, max_tokens):
    rng = np.random.default_rng(seed)
    ops = []
    if preload:
        ops.append(("preload", [int(e) for e in rng.permutation(E)[: S + 3]]))
    p = 1.0 / np.arange(1, E + 1) ** 1.2
    p = p[rng.permutation(E)]
    p /= p.sum()
    for step in range(steps):
        T = int(rng.integers(1, max_tokens + 1))
        needed = np.unique(np.concatenate([rng.choice(E, 8, replace=False, p=p) for _ in range(T)]))
        needed = rng.permutation(needed)[:S]                 # any order, never more than S
        ops.append(("resolve", [int(e) for e in needed], bool(step % 3), bool(step % 4)))
        if step % 16 == 15:
            ops.append(("decay",))
    return ops


@pytest.mark.parametrize("seed,S,E,preload,max_tokens", [(11, 64, 256, True, 1), (12, 96, 256, False, 4),
                                                          (13, 16, 64, True, 2), (14, 200, 256, True, 8),
                                                          (15, 8, 32, False, 1)])
def test_native_table_equals_the_oracle(seed, S, E, preload, max_tokens):
    import mimo_moe
    nat, ora = mimo_moe.SlotCache(S, E), OracleSlotCache(S, E)
    for op in _sequence(seed, S, E, 250, preload, max_tokens):
        if op[0] == "preload":
            assert nat.preload(op[1]) == ora.preload(op[1])
        elif op[0] == "decay":
            nat.decay()
            ora.decay()
        else:
            assert nat.resolve(op[1], op[2], op[3]) == ora.resolve(op[1], op[2], op[3])
        assert np.array_equal(nat.slot_of, ora.slot_of) and np.array_equal(nat.expert_in, ora.expert_in)
        assert (nat.hits, nat.misses) == (ora.hits, ora.misses)


def test_native_table_rejects_what_it_cannot_hold():
    """A step needing more distinct experts than slots: ValueError and nothing changed (the reference raises
    only when the missing experts alone are more, and can otherwise evict one of the step's own experts,
    which the oracle keeps); repeated or out-of-range ids and bad sizes: ValueError."""
    import mimo_moe
    with pytest.raises(ValueError):
        mimo_moe.SlotCache(0, 256)
    with pytest.raises(ValueError):
        mimo_moe.SlotCache(300, 256)
    nat, ora = mimo_moe.SlotCache(4, 16), OracleSlotCache(4, 16)
    assert nat.preload([3, 5]) == ora.preload([3, 5]) == [(3, 0), (5, 1)]
    before = (nat.slot_of.copy(), nat.expert_in.copy(), nat.hits, nat.misses)
    with pytest.raises(ValueError):
        nat.resolve([3, 5, 7, 8, 9])                     # 5 distinct experts, 4 slots, 3 missing
    assert np.array_equal(nat.slot_of, before[0]) and np.array_equal(nat.expert_in, before[1])
    assert (nat.hits, nat.misses) == before[2:]
    loads = ora.resolve([3, 5, 7, 8, 9])                 # the reference's rule: allowed, evicts a needed expert
    assert len(loads) == 3 and (ora.slot_of[[3, 5, 7, 8, 9]] < 0).sum() == 1
    for bad in ([3, 3], [16], [-1]):
        with pytest.raises(ValueError):
            nat.resolve(bad)
    # the table still follows the oracle after the rejected calls (the oracle never saw them)
    ora2 = OracleSlotCache(4, 16)
    ora2.preload([3, 5])
    for needed in ([1, 2], [3, 4, 6], [7], [2, 5, 9, 10]):
        assert nat.resolve(needed) == ora2.resolve(needed)
    assert np.array_equal(nat.slot_of, ora2.slot_of)


def test_preload_on_a_filled_table_stays_consistent():
    import mimo_moe
    nat = mimo_moe.SlotCache(4, 16)
    nat.preload([1, 2, 3, 4])
    nat.preload([4, 9])                                   # 4 moves to slot 0, 1 and 9's old slots are unmapped
    so, ei = nat.slot_of, nat.expert_in
    assert list(ei) == [4, 9, 3, -1]
    assert so[4] == 0 and so[9] == 1 and so[3] == 2 and so[1] == -1 and so[2] == -1
    assert all(so[e] == s for s, e in enumerate(ei) if e >= 0)


def test_fixture_regenerates_from_the_reference():
    """Where the reference checkout is present (the build's reference root), its own SlotCache, loaded by path
    and run unchanged, reproduces the committed runs exactly."""
    import importlib.util
    from __graft_entry__ import REFERENCE_ROOT
    if not (REFERENCE_ROOT / "engine" / "mimo_stream" / "cache.py").exists():
        pytest.skip("reference checkout not present")
    spec = importlib.util.spec_from_file_location("make_slot_cache_golden", GOLDEN.with_name("make_slot_cache_golden.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    assert json.loads(json.dumps(gen.runs(gen.reference_slot_cache(str(REFERENCE_ROOT))))) == _runs()
