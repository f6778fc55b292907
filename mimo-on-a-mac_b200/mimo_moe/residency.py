"""Expert residency: a layer's experts in host memory, S of them resident in device slots.

The reference keeps S experts per layer resident in unified memory and streams the rest from SSD when a
step needs them (engine/mimo_stream/cache.py:13-65, the slot table; model.py:130-167, the per-layer banks
and warm-up; model.py:184-222, a step: resolve the routed experts, read the misses into their slots,
group the routes by slot and run the expert kernels on the bank).  On B200 all 48 layers' experts
(164 GB) fit in HBM, so the engine path keeps every expert resident; this module is for the cases that do
not fit (a longer model, several models on one GPU, a smaller device): the experts live in pinned host
memory and the misses cross to the slots by host->device copies.

SlotCache is the reference's table over the library's native one (mimo_moe_slot_cache_*).  ExpertCache
runs one MoE layer from a slot bank: route on the device, one host sync on the routes (model.py:315-323),
resolve, copy the loaded experts into their slots on the stream, then the same kernels as the resident
path through the slot map (decode: routes grouped by slot, model.py:217-219; prefill: mimo_moe_prefill's
slot_of), so its output equals the resident block's on the same routes bit for bit.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .ops import TOPK, ExpertPools, _status, group_routes, moe_experts, moe_prefill, read_status, router

DECODE_DECAY_EVERY = 16   # model.py:348-354: counts halve every 16 decode tokens


class SlotCache:
    """Drop-in for engine/mimo_stream/cache.py SlotCache (preload, resolve, decay, slot_of, expert_in, hits,
    misses), over the native table.  resolve() raises ValueError when the step needs more distinct experts
    than there are slots (the reference: when the missing ones alone are more)."""

    def __init__(self, n_slots: int, n_experts: int = 256):
        h = lib().mimo_moe_slot_cache_create(int(n_slots), int(n_experts))
        if not h:
            raise ValueError(f"bad slot table size: {n_slots} slots for {n_experts} experts")
        self._h = ctypes.c_void_p(h)
        self.S, self.E = int(n_slots), int(n_experts)
        self._le = np.empty(self.S, np.int32)
        self._ls = np.empty(self.S, np.int32)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            self._h = None
            try:
                lib().mimo_moe_slot_cache_destroy(h)
            except Exception:   # interpreter shutdown: the library may already be gone
                pass

    @staticmethod
    def _ids(ids) -> np.ndarray:
        return np.ascontiguousarray(np.asarray(ids, dtype=np.int64).reshape(-1).astype(np.int32))

    def _loads(self, n: int) -> List[Tuple[int, int]]:
        return [(int(e), int(s)) for e, s in zip(self._le[:n], self._ls[:n])]

    def preload(self, experts: Sequence[int]) -> List[Tuple[int, int]]:
        ids = self._ids(list(experts)[: self.S])
        n = ctypes.c_int32(0)
        check(lib().mimo_moe_slot_cache_preload(self._h, ids.ctypes.data, ids.size, self._le.ctypes.data,
                                                self._ls.ctypes.data, ctypes.byref(n)), "slot_cache_preload")
        return self._loads(n.value)

    def resolve(self, needed, count: bool = True, stats: bool = True) -> List[Tuple[int, int]]:
        ids = self._ids(needed)
        n = ctypes.c_int32(0)
        rc = lib().mimo_moe_slot_cache_resolve(self._h, ids.ctypes.data, ids.size, int(count), int(stats),
                                               self._le.ctypes.data, self._ls.ctypes.data, ctypes.byref(n))
        if rc == _lib.MIMO_ERANGE:
            raise ValueError("step needs more distinct experts than the pool holds")
        check(rc, "slot_cache_resolve")
        return self._loads(n.value)

    def decay(self) -> None:
        check(lib().mimo_moe_slot_cache_decay(self._h), "slot_cache_decay")

    def _state(self):
        slot_of = np.empty(self.E, np.int32)
        expert_in = np.empty(self.S, np.int32)
        hits, misses = ctypes.c_int64(0), ctypes.c_int64(0)
        check(lib().mimo_moe_slot_cache_state(self._h, slot_of.ctypes.data, expert_in.ctypes.data,
                                              ctypes.byref(hits), ctypes.byref(misses)), "slot_cache_state")
        return slot_of, expert_in, hits.value, misses.value

    @property
    def slot_of(self) -> np.ndarray:
        return self._state()[0]

    @property
    def expert_in(self) -> np.ndarray:
        return self._state()[1]

    @property
    def hits(self) -> int:
        return self._state()[2]

    @property
    def misses(self) -> int:
        return self._state()[3]


class ExpertCache:
    """One MoE layer whose E experts live in host memory (the reference layout, `host` = {gate,up,down}_{w,s}
    CPU tensors with E experts each; pinned here if they are not) with `n_slots` of them resident on
    `device`.  __call__(x, router_w, bias) -> y bf16 [T, H], the reference's per-layer step
    (model.py:184-222 decode / verify); a prefill step (T > 8) also makes every routed expert resident
    through the table, where the reference's _moe_prefill (model.py:230-285) leaves the table alone and
    streams the non-resident experts through staging banks.  A step raises ValueError when it routes to
    more distinct experts than there are slots.  Every DECODE_DECAY_EVERY single-token calls the counts
    decay (model.py:348-354)."""

    def __init__(self, host: Dict[str, torch.Tensor], n_slots: int, device=None, topk: int = TOPK):
        self.host = {}
        for k in ExpertPools.KEYS:
            t = host[k]
            if t.is_cuda:
                raise ValueError(f"{k}: the experts' home is host memory")
            t = t.contiguous()
            self.host[k] = t if t.is_pinned() else t.pin_memory()
        gw = self.host["gate_w"]
        self.E, inter, hidden = gw.shape[0], gw.shape[1], gw.shape[2] * 8
        self.device = torch.device(device or "cuda")
        self.pools = ExpertPools.empty(n_slots, hidden, inter, self.device)
        self.table = SlotCache(n_slots, self.E)
        self.topk = topk
        self.decode_calls = 0
        self.copied_bytes = 0
        self._slot_of_host = torch.empty(self.E, dtype=torch.int32).pin_memory()
        self._map_copied = torch.cuda.Event()
        self.slot_of = torch.full((self.E,), -1, dtype=torch.int32, device=self.device)

    @property
    def S(self) -> int:
        return self.pools.S

    def _copy_in(self, loads: List[Tuple[int, int]]) -> None:
        """Host -> slot copies of the loaded experts, in stream order after the kernels that last read the
        victim slots (the routes' host sync already waited for them), then the new slot map."""
        for e, s in loads:
            for k in ExpertPools.KEYS:
                self.pools.t[k][s].copy_(self.host[k][e], non_blocking=True)
                self.copied_bytes += self.host[k][e].numel() * self.host[k][e].element_size()
        if loads:
            self._map_copied.synchronize()   # the staging buffer's previous copy has left it
            self._slot_of_host.copy_(torch.from_numpy(self.table.slot_of))
            self.slot_of.copy_(self._slot_of_host, non_blocking=True)
            self._map_copied.record()

    def warm(self, experts: Optional[Sequence[int]] = None) -> None:
        """Fill the slots (model.py:159-167): the given experts (e.g. by profile frequency), else 0..S-1."""
        order = list(range(self.E)) if experts is None else list(experts)
        self._copy_in(self.table.preload(order[: self.S]))

    def ensure(self, needed) -> List[Tuple[int, int]]:
        """Make the distinct experts `needed` resident; returns the (expert, slot) loads it copied."""
        loads = self.table.resolve(needed)
        self._copy_in(loads)
        return loads

    def __call__(self, x: torch.Tensor, router_w: torch.Tensor, bias: Optional[torch.Tensor] = None,
                 status: Optional[torch.Tensor] = None, return_routes: bool = False):
        if router_w.shape[0] != self.E:
            raise ValueError(f"router has {router_w.shape[0]} experts, the cache {self.E}")
        x = x.to(device=self.device, dtype=torch.bfloat16).contiguous()
        T = x.shape[0]
        idx, w = router(x, router_w, bias, self.topk)
        self.ensure(np.unique(idx.cpu().numpy()))          # the per-layer host sync of the reference
        st = _status(self.device) if status is None else status
        if T <= 8:
            slot_idx = self.slot_of[idx.long()]
            g = group_routes(slot_idx, w, R=8, E=self.S)
            y = moe_experts(x, self.pools, g.uids, g.urows, g.ucnt, g.uw, R=g.R, gather_idx=g.gather_idx,
                            num_unique=g.num_unique, pairs_rounding=T == 1, status=st)
        else:
            y = moe_prefill(x, self.pools, idx, w, slot_of=self.slot_of, E=self.E, status=st)
        if status is None:
            read_status(st, "expert cache step")
        if T == 1:
            self.decode_calls += 1
            if self.decode_calls % DECODE_DECAY_EVERY == 0:
                self.table.decay()
        return (y, idx, w) if return_routes else y
