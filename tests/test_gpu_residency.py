"""The expert residency path on the GPU (mimo_moe.ExpertCache: a layer's experts in pinned host memory, S of them
in device slots, engine/mimo_stream/model.py:184-222): every step equal, bit for bit, to the resident pool's
kernels on the same routes (decode: routes grouped by slot; prefill: slot_of), the slot table's loads copied
into their slots, and a step routed to more distinct experts than slots refused before any launch."""
import numpy as np
import pytest
import torch

from oracle import synth

pytestmark = pytest.mark.gpu

E = 64


@pytest.fixture(scope="module")
def layer(gpu):
    import mimo_moe
    pool = mimo_moe.ExpertPools.synthetic(E, seed=0, layer=2, device=gpu)
    host = {k: v.cpu().pin_memory() for k, v in pool.t.items()}
    W = synth.router_weight(E).to(gpu)
    return pool, host, W


def _resident(pool, x, idx, w):
    import mimo_moe
    if x.shape[0] <= 8:
        g = mimo_moe.group_routes(idx, w, R=8, E=pool.S)
        return mimo_moe.moe_experts(x, pool, g.uids, g.urows, g.ucnt, g.uw, R=8, gather_idx=g.gather_idx,
                                    num_unique=g.num_unique, pairs_rounding=x.shape[0] == 1)
    return mimo_moe.moe_prefill(x, pool, idx, w)


def _same(a, b):
    return torch.equal(a.view(torch.int16), b.view(torch.int16))


def _expert_bytes(host):
    return sum(v[0].numel() * v[0].element_size() for v in host.values())


def test_decode_steps_from_a_slot_bank_equal_the_resident_kernels(gpu, layer):
    import mimo_moe
    pool, host, W = layer
    S = 40
    cache = mimo_moe.ExpertCache(host, S, device=gpu)
    cache.warm(list(range(E - 1, E - 1 - S, -1)))      # experts 63..24, in reverse order over the slots
    assert cache.copied_bytes == S * _expert_bytes(host)
    Ts = [1, 2, 4, 1, 3, 1, 1, 2, 4, 1, 1, 1, 1, 1, 1, 1, 1, 1, 4, 1]
    distinct = 0
    for i, T in enumerate(Ts):
        x = synth.hidden(T, seed=300 + i).to(gpu)
        y, idx, w = cache(x, W, None, return_routes=True)
        assert _same(y, _resident(pool, x, idx, w)), f"step {i} (T={T})"
        distinct += np.unique(idx.cpu().numpy()).size
    t = cache.table
    assert t.hits + t.misses == distinct and t.misses > 0
    assert cache.copied_bytes == (S + t.misses) * _expert_bytes(host)
    assert cache.decode_calls == Ts.count(1)
    so, ei = t.slot_of, t.expert_in
    assert all(so[e] == s for s, e in enumerate(ei) if e >= 0)
    assert torch.equal(cache.slot_of.cpu(), torch.from_numpy(so))
    for s in (0, 17, S - 1):                             # the slots hold their experts' bytes
        e = int(ei[s])
        for k in mimo_moe.ExpertPools.KEYS:
            assert torch.equal(cache.pools.t[k][s].cpu(), host[k][e])


def test_prefill_from_a_slot_bank_equals_the_resident_kernels(gpu, layer):
    import mimo_moe
    pool, host, W = layer
    cache = mimo_moe.ExpertCache(host, E, device=gpu)
    perm = np.random.default_rng(5).permutation(E)
    cache.warm([int(e) for e in perm[:48]])               # 48 experts in shuffled slots, 16 slots empty
    distinct = 0
    for i, T in enumerate([12, 40]):
        x = synth.hidden(T, seed=400 + i).to(gpu)
        y, idx, w = cache(x, W, None, return_routes=True)
        assert _same(y, _resident(pool, x, idx, w)), f"T={T}"
        distinct += np.unique(idx.cpu().numpy()).size
    assert cache.table.hits + cache.table.misses == distinct


def test_a_step_beyond_the_slots_is_refused(gpu, layer):
    import mimo_moe
    pool, host, W = layer
    cache = mimo_moe.ExpertCache(host, 16, device=gpu)
    x = synth.hidden(8, seed=500).to(gpu)
    idx, _ = mimo_moe.router(x, W, None)
    assert np.unique(idx.cpu().numpy()).size > 16
    with pytest.raises(ValueError):
        cache(x, W)
    assert cache.table.hits == cache.table.misses == 0 and cache.copied_bytes == 0
