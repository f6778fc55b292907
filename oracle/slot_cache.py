"""CPU oracle for the expert residency cache: the per-layer slot table with decayed-LFU eviction of
engine/mimo_stream/cache.py:13-65.

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library imports this module: `tests/` use it as the
checker of the library's native slot table (mimo_moe_slot_cache_*).

The policy, restated (cache.py line numbers):
  * preload(experts) (24-28): the first S experts go to slots 0, 1, ... in order; returns (expert, slot).
  * resolve(needed, count, stats) (30-62), `needed` distinct expert ids:
      t += 1; cnt[needed] += 1 when count; last[needed] = t;
      missing = the needed experts without a slot, in `needed` order;
      hits += |needed| - |missing|, misses += |missing| when stats;
      more missing than slots raises ValueError;
      score of a slot = cnt[e] * 1e12 + last[e] for its expert e, -1 for an empty slot, +inf for a slot
      holding a needed expert; the |missing| lowest-scoring slots are the victims; missing[i] moves into
      victims[i] (the victim's expert loses its slot).
  * decay() (64-65): cnt *= 0.5 (the engine calls it every 16 decode tokens, model.py:348-354).

The reference picks the victims with np.argpartition, which leaves the order of the victims and the choice
among equal scores unspecified.  This restatement fixes both: victims in ascending (score, slot) order.
tests/test_slot_cache.py pins everything else to the reference's own class through recorded runs of it
(tests/golden/slot_cache.json): the same missing experts, hit and miss counts at every step, and victim
scores equal as multisets.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import numpy as np


class SlotCache:
    def __init__(self, n_slots: int, n_experts: int = 256):
        self.S = n_slots
        self.slot_of = np.full(n_experts, -1, np.int32)   # expert -> slot or -1
        self.expert_in = np.full(n_slots, -1, np.int32)   # slot -> expert or -1
        self.cnt = np.zeros(n_experts, np.float64)
        self.last = np.zeros(n_experts, np.int64)
        self.t = 0
        self.hits = 0
        self.misses = 0
        self.scores: Optional[np.ndarray] = None          # the slot scores of the last resolve with misses

    def preload(self, experts: Sequence[int]) -> List[Tuple[int, int]]:
        experts = [int(e) for e in list(experts)[: self.S]]
        for s, e in enumerate(experts):
            self.slot_of[e] = s
            self.expert_in[s] = e
        return list(zip(experts, range(len(experts))))

    def resolve(self, needed, count: bool = True, stats: bool = True,
                victims: Optional[Sequence[int]] = None) -> List[Tuple[int, int]]:
        """`victims`, when given, replaces the oracle's own choice (a test replays another implementation's
        choice among equal scores with it)."""
        self.t += 1
        needed = np.asarray(needed, np.int64)
        if count:
            self.cnt[needed] += 1
        self.last[needed] = self.t
        missing = needed[self.slot_of[needed] < 0]
        if stats:
            self.hits += len(needed) - len(missing)
            self.misses += len(missing)
        if len(missing) == 0:
            return []
        if len(missing) > self.S:
            raise ValueError("step needs more distinct experts than the pool holds")
        exp = self.expert_in
        e0 = np.maximum(exp, 0)
        score = np.where(exp >= 0, self.cnt[e0] * 1e12 + self.last[e0], -1.0)
        held = self.slot_of[needed]
        score[held[held >= 0]] = np.inf
        self.scores = score.copy()
        if victims is None:
            victims = np.lexsort((np.arange(self.S), score))[: len(missing)]
        loads = []
        for e, s in zip(missing, victims):
            old = exp[s]
            if old >= 0:
                self.slot_of[old] = -1
            exp[s] = e
            self.slot_of[e] = s
            loads.append((int(e), int(s)))
        return loads

    def decay(self) -> None:
        self.cnt *= 0.5
