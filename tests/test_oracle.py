"""CPU checks of the oracle itself (no GPU): MXFP4 decode semantics, routing order, grouping and
permutation rules, the synthetic generator, and the reference test's accuracy / negative-control
figures (engine/tests/test_kernels.py:65-89, bench/reports/kernels.md:10-16)."""
import numpy as np
import pytest

from oracle import mimo_oracle as O
from oracle import synth


def test_e2m1_and_e8m0_decode():
    # kernels.py:21-29: e2m1 magnitude table, sign bit 3; e8m0 2^(s-127), 0 -> 2^-127, 255 -> NaN
    codes = np.arange(16, dtype=np.uint32)
    words = (codes[None, :] << (4 * np.arange(8, dtype=np.uint32)[:, None])).T.copy()  # code in nibble j
    vals = O.unpack_e2m1(words)          # [16, 64]
    for c in range(16):
        row = vals[c].reshape(8, 8)
        assert np.all(row[np.arange(8), np.arange(8)] == O.E2M1[c])
    assert list(O.E2M1[:8]) == [0, 0.5, 1, 1.5, 2, 3, 4, 6]
    s = O.e8m0_to_f32(np.array([0, 1, 127, 128, 254, 255], np.uint8))
    assert s[0] == np.float32(2.0 ** -127) and s[1] == np.float32(2.0 ** -126)
    assert s[2] == 1.0 and s[3] == 2.0 and s[4] == np.float32(2.0 ** 127) and np.isnan(s[5])
    w = np.random.default_rng(0).integers(0, 2 ** 32, size=(3, 16), dtype=np.uint32)
    sc = np.random.default_rng(1).integers(100, 140, size=(3, 4), dtype=np.uint8)
    assert np.array_equal(O.dequant64(w, sc), O.dequant(w, sc).astype(np.float64))


def test_low_nibble_first():
    w = np.array([[0x76543210]], np.uint32)
    assert list(O.unpack_e2m1(w)[0]) == [0, 0.5, 1, 1.5, 2, 3, 4, 6]


def test_bf16_rounding_is_rne():
    a = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 1.0 + 2 ** -8 + 2 ** -20, -2.5, np.nan], np.float32)
    r = O.bf16_round(a)
    assert r[0] == 1.0 and r[1] == 1.0 + 2 ** -6 and r[2] == 1.0 + 2 ** -7 and r[3] == -2.5
    assert np.isnan(r[4])


def test_topk_total_order_ties_and_nan():
    logits = np.zeros((2, 256), np.float32)
    logits[0, [5, 9, 200]] = 3.0          # exact ties -> ascending id
    logits[0, 17] = np.nan                # NaN ranks last
    logits[1] = np.linspace(-4, 4, 256, dtype=np.float32)
    inds, w = O.topk_from_logits(logits, np.zeros(256, np.float32))
    assert list(inds[0, :3]) == [5, 9, 200]
    assert 17 not in inds[0]
    assert list(inds[1]) == list(range(255, 247, -1))
    s = O.sigmoid_f32(logits[1, inds[1]])
    tot = np.float32(0)
    for v in s:
        tot = np.float32(tot + v)
    tot = np.float32(tot + np.float32(1e-20))
    assert np.array_equal(w[1], (s / tot).astype(np.float32))


def test_bias_changes_selection_not_weights():
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((4, 256)).astype(np.float32)
    bias = np.zeros(256, np.float32)
    bias[:8] = 10.0
    inds, w = O.topk_from_logits(logits, bias)
    assert (np.sort(inds, axis=1) == np.arange(8)).all()
    s = O.sigmoid_f32(logits[:, :8])
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)
    assert np.allclose(np.sort(w, 1), np.sort(s / s.sum(1, keepdims=True), 1), rtol=1e-6)


def test_group_routes_rules():
    inds = np.array([[3, 1, 7, 2], [1, 3, 9, 4]])
    sc = np.arange(8, dtype=np.float32).reshape(2, 4) / 10
    uids, urows, ucnt, uw, gidx = O.group_routes(inds, sc, R=8)
    assert list(uids) == [1, 2, 3, 4, 7, 9]
    assert list(ucnt) == [2, 1, 2, 1, 1, 1]
    assert list(urows[0, :2]) == [0, 1] and list(uw[0, :2]) == [np.float32(0.1), np.float32(0.4)]
    assert list(gidx) == [2 * 8, 0, 4 * 8, 1 * 8, 0 * 8 + 1, 2 * 8 + 1, 5 * 8, 3 * 8]
    with pytest.raises(ValueError):
        O.group_routes(np.zeros((3, 1), np.int64), np.ones((3, 1), np.float32), R=2)


def test_dispatch_is_stable_argsort():
    rng = np.random.default_rng(1)
    inds = rng.integers(0, 256, size=(300, 8))
    off, order, inv = O.dispatch(inds)
    flat = inds.reshape(-1)
    assert np.all(np.diff(flat[order]) >= 0)
    for e in (0, 17, 255):
        pos = order[off[e]:off[e + 1]]
        assert np.all(np.diff(pos) > 0) and np.all(flat[pos] == e)
    assert np.array_equal(inv[order], np.arange(order.size))


def test_synth_distribution():
    w = synth.expert_tensor(0, 0, "gate_w", 3, (2048, 4096))
    s = synth.expert_tensor(0, 0, "gate_s", 3, (2048, 4096))
    assert w.shape == (2048, 512) and s.shape == (2048, 128)
    nib = (w[..., None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF
    counts = np.bincount(nib.reshape(-1), minlength=16)
    assert counts.min() > 0.97 * counts.mean() and counts.max() < 1.03 * counts.mean()
    assert set(np.unique(s)) == {119, 120}
    assert abs((s == 120).mean() - 0.6875) < 0.01
    d = O.dequant(w, s)
    assert abs(d.std() - 0.02) < 0.001
    assert not np.array_equal(w, synth.expert_tensor(0, 0, "gate_w", 4, (2048, 4096)))
    assert not np.array_equal(w, synth.expert_tensor(0, 1, "gate_w", 3, (2048, 4096)))
    assert not np.array_equal(w, synth.expert_tensor(0, 0, "up_w", 3, (2048, 4096)))


def small_pool(S, seed=0, H=512, I=256):
    shapes = {"gate": (I, H), "up": (I, H), "down": (H, I)}
    sp = synth.SynthPool(seed, 0, shapes)
    return {f"{n}_{k}": np.stack([sp[f"{n}_{k}"][e] for e in range(S)]) for n in shapes for k in "ws"}


def test_kernel_math_accuracy_and_negative_control():
    """The reference reports 0.40-0.45% max rel err of its kernels vs FP32 dequant and 130% for a
    nibble-order swap (bench/reports/kernels.md:10-16); the restated kernel math must land in the
    same band, and the swapped-nibble control must fail."""
    S, H = 24, 512
    arrays = small_pool(S, H=H, I=256)
    pool = O.Pool(arrays, cache=S)
    rng = np.random.default_rng(0)
    for M in (1, 4, 8):
        x = O.bf16_round(rng.standard_normal((M, H)).astype(np.float32))
        inds = np.stack([rng.choice(S, 8, replace=False) for _ in range(M)])
        if M > 1:
            inds[1, :4] = inds[0, :4]
        sc = rng.random((M, 8)).astype(np.float32)
        sc /= sc.sum(1, keepdims=True)
        ref = O.reference_fp32(x, pool, inds, sc)
        y = O.moe_layer(x, pool, inds, sc)
        e = O.rel_err(y, ref)
        assert 1e-4 < e < 1e-2, (M, e)
        uids, urows, ucnt, uw, gidx = O.group_routes(inds, sc)
        yg = O.moe_experts(x, pool, uids, urows, ucnt, uw, gather_idx=gidx)
        assert O.rel_err(yg, ref) < 1e-2
    sw = dict(arrays)
    for n in ("gate", "up", "down"):
        w = arrays[f"{n}_w"]
        sw[f"{n}_w"] = ((w & 0x0F0F0F0F) << 4) | ((w >> 4) & 0x0F0F0F0F)
    bad = O.Pool(sw, cache=S)
    x = O.bf16_round(rng.standard_normal((4, H)).astype(np.float32))
    inds = np.stack([rng.choice(S, 8, replace=False) for _ in range(4)])
    sc = np.full((4, 8), 1 / 8, np.float32)
    assert O.rel_err(O.moe_layer(x, bad, inds, sc), O.reference_fp32(x, pool, inds, sc)) > 0.5


def test_package_input_generators_match_the_oracle_fixtures():
    """bench.py draws its inputs from mimo_moe.synthetic; the oracle's generators (which the parity
    tests and golden fixtures use) must give the same tensors bit for bit."""
    import torch
    from mimo_moe import synthetic
    assert torch.equal(synthetic.hidden(5, seed=1234).view(torch.int16), synth.hidden(5, seed=1234).view(torch.int16))
    assert torch.equal(synthetic.router_weight(E=64).view(torch.int16), synth.router_weight(E=64).view(torch.int16))
    for c in (1.0, 0.055):
        assert torch.equal(synthetic.zipf_bias(c=c), synth.zipf_bias(c=c))
    assert torch.equal(synthetic.overlap_bias(), synth.overlap_bias())


def test_rmsnorm_oracle_properties():
    """Unit RMS after the norm, invariance under power-of-two scaling (eps 0: every step scales
    exactly), the weight as a bf16 multiply of the normalised row, zero rows stay zero."""
    rng = np.random.default_rng(4)
    x = O.bf16_round(rng.standard_normal((6, 4096)).astype(np.float32))
    y = O.rmsnorm(x)
    assert np.allclose(np.sqrt((y.astype(np.float64) ** 2).mean(-1)), 1.0, atol=4e-3)
    assert np.array_equal(O.rmsnorm(x, eps=0.0), O.rmsnorm(x * np.float32(64), eps=0.0))
    w = O.bf16_round(rng.standard_normal(4096).astype(np.float32))
    assert np.array_equal(O.rmsnorm(x, w), O.bf16_round(w * y))
    assert np.array_equal(O.rmsnorm(np.zeros((1, 64), np.float32)), np.zeros((1, 64), np.float32))


def test_batched_pair_path_equals_the_oracle_bit_for_bit():
    """oracle/batched.py (torch, one float64 product per expert, used for the GPU checks at the BASELINE.json sizes)
    against mimo_oracle.moe_pairs on full-size experts: every output bit equal, with a slot map, shared
    experts across rows and the M = 1 case."""
    import torch
    from oracle import batched as B
    sp = synth.SynthPool(0, 6)
    S = 4
    pool = {n: torch.from_numpy(np.stack([sp[n][e] for e in range(S)]).view(np.int32 if n.endswith("_w") else np.uint8))
            for n in ("gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")}
    rng = np.random.default_rng(12)
    for T, k in ((1, 3), (9, 3)):
        x = synth.hidden(T, seed=60 + T).float().numpy()
        inds = np.stack([rng.choice(S, k, replace=False) for _ in range(T)]).astype(np.int32)
        w = rng.random((T, k)).astype(np.float32)
        want = O.moe_pairs(x, O.Pool(sp, cache=S), inds, w)
        assert np.array_equal(B.moe_pairs(x, pool, inds, w).view(np.uint32), want.view(np.uint32))
        experts = np.array([200, 7, 31, 90])               # expert ids -> slots through slot_of
        slot_of = np.full(256, -1, np.int32)
        slot_of[experts] = np.arange(S)
        got = B.moe_pairs(x, pool, experts[inds], w, slot_of=slot_of)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # the distinct-expert path (2 <= T <= 8): route-order combine and the scatter-add order
    x = synth.hidden(5, seed=71).float().numpy()
    inds = np.stack([rng.choice(S, 3, replace=False) for _ in range(5)]).astype(np.int32)
    w = rng.random((5, 3)).astype(np.float32)
    opool = O.Pool(sp, cache=S)
    assert np.array_equal(B.moe_layer(x, pool, inds, w).view(np.uint32), O.moe_layer(x, opool, inds, w, R=8).view(np.uint32))
    uids, urows, ucnt, uw, _ = O.group_routes(inds, w)
    want = O.moe_experts(x, opool, uids, urows, ucnt, uw, gather_idx=None)
    assert np.array_equal(B.moe_grouped(x, pool, inds, w, unit_order=True).view(np.uint32), want.view(np.uint32))


def test_overlap_bias_gives_the_config1_expert_sharing():
    """BASELINE.json config 1's forced-overlap variant: consecutive rows of the seeded 8-row decode batches share
    2.6 +- 0.1 of their 8 experts under synth.overlap_bias() (free routing shares ~0.25)."""
    W = synth.router_weight().float().numpy()
    b = synth.overlap_bias().numpy()
    shared = []
    for i in range(16):
        inds, _ = O.topk_from_logits(O.router_logits(synth.hidden(8, seed=2 + 1000 * i).float().numpy(), W), b)
        shared += [len(set(inds[t]) & set(inds[t + 1])) for t in range(7)]
    assert abs(np.mean(shared) - 2.6) <= 0.1, np.mean(shared)
