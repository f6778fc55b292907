"""GPU parity of every stage against the CPU oracle, through the C ABI (libmimo_moe.so).

Bars: bit-exact for top-k indices / weights (given identical logits), route grouping and the prefill
permutation; rel_err = max|a-b| / max|b| (engine/tests/test_kernels.py:54-56) <= 1e-2 for outputs
against the bf16-faithful oracle, and < 2e-2 against the FP32 dequant reference (the reference test's
own threshold, test_kernels.py:79,89)."""
import numpy as np
import pytest
import torch

from oracle import mimo_oracle as O
from oracle import synth

pytestmark = pytest.mark.gpu

TOL_ORACLE = 1e-2   # vs the bf16-faithful restatement of the reference path
TOL_FP32 = 2e-2     # vs FP32 dequant (the reference test's bar)


def f32(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(scope="module")
def pool24(gpu):
    import mimo_moe
    p = mimo_moe.ExpertPools.synthetic(24, seed=0, layer=0, device=gpu)
    torch.cuda.synchronize()
    return p, O.Pool(synth.SynthPool(0, 0), cache=24)


def test_synthetic_pool_matches_numpy_generator(gpu):
    import mimo_moe
    p = mimo_moe.ExpertPools.synthetic(3, seed=7, layer=5, first_expert=40, device=gpu)
    for name, shp in (("gate_w", (2048, 4096)), ("up_s", (2048, 4096)), ("down_w", (4096, 2048)),
                      ("down_s", (4096, 2048))):
        got = p[name][2].cpu().numpy().view(np.uint32 if name.endswith("_w") else np.uint8)
        want = synth.expert_tensor(7, 5, name, 42, shp)
        assert np.array_equal(got, want), name


def test_topk_bit_exact_given_logits(gpu):
    import mimo_moe
    rng = np.random.default_rng(3)
    logits = rng.standard_normal((257, 256)).astype(np.float32) * 3
    logits[0, [1, 2, 3, 40, 41]] = 2.5           # exact ties
    logits[1, :] = 30.0                          # sigmoid saturates to 1.0: ties everywhere
    logits[2, 7] = np.nan
    logits[3, :20] = -np.inf
    bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
    bias[:16] = 0.0
    for b in (None, bias):
        idx, w = mimo_moe.topk(torch.from_numpy(logits).to(gpu), None if b is None else torch.from_numpy(b).to(gpu))
        ri, rw = O.topk_from_logits(logits, np.zeros(256, np.float32) if b is None else b)
        assert np.array_equal(idx.cpu().numpy(), ri)
        assert np.array_equal(w.cpu().numpy().view(np.uint32), rw.view(np.uint32))


def test_router_logits_and_selection(gpu):
    import mimo_moe
    for T in (1, 8, 300):
        x = synth.hidden(T)
        W = synth.router_weight()
        bias = synth.overlap_bias() if T == 8 else torch.zeros(256)
        idx, w, logits = mimo_moe.router(x.to(gpu), W.to(gpu), bias.to(gpu), return_logits=True)
        ref = O.router_logits(x.float().numpy(), W.float().numpy())
        got = logits.cpu().numpy()
        scale = np.abs(x.float().numpy()) @ np.abs(W.float().numpy()).T
        assert np.all(np.abs(got - ref) <= 1e-5 * scale + 1e-6)
        ri, rw = O.topk_from_logits(got, bias.numpy())        # bit-exact given the same logits
        assert np.array_equal(idx.cpu().numpy(), ri)
        assert np.array_equal(w.cpu().numpy().view(np.uint32), rw.view(np.uint32))


@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_group_routes_bit_exact(gpu, M):
    import mimo_moe
    rng = np.random.default_rng(M)
    inds = np.stack([rng.choice(256, 8, replace=False) for _ in range(M)]).astype(np.int32)
    if M > 1:
        inds[1, :4] = inds[0, :4]
    sc = rng.random((M, 8)).astype(np.float32)
    g = mimo_moe.group_routes(torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu), check_rows=True)
    uids, urows, ucnt, uw, gidx = g.trimmed()
    r = O.group_routes(inds, sc, R=8)
    assert np.array_equal(uids.numpy(), r[0]) and np.array_equal(urows.numpy(), r[1])
    assert np.array_equal(ucnt.numpy(), r[2]) and np.array_equal(uw.numpy(), r[3])
    assert np.array_equal(gidx.numpy(), r[4].astype(np.int32))


def test_group_routes_overflow_raises_like_reference(gpu):
    import mimo_moe
    inds = torch.zeros(3, 1, dtype=torch.int32, device=gpu)
    with pytest.raises(ValueError):
        mimo_moe.group_routes(inds, torch.ones(3, 1, device=gpu), R=2, check_rows=True)


@pytest.mark.parametrize("T,skew", [(1, False), (37, False), (2048, False), (2048, True), (16384, True)])
def test_dispatch_bit_exact(gpu, T, skew):
    import mimo_moe
    rng = np.random.default_rng(T)
    if skew:
        p = 1.0 / np.arange(1, 257) ** 1.1
        inds = np.stack([rng.choice(256, 8, replace=False, p=p / p.sum()) for _ in range(T)]).astype(np.int32)
    else:
        inds = np.stack([rng.choice(256, 8, replace=False) for _ in range(T)]).astype(np.int32)
    off, order, inv = mimo_moe.dispatch(torch.from_numpy(inds).to(gpu))
    ro, rord, rinv = O.dispatch(inds)
    assert np.array_equal(off.cpu().numpy(), ro)
    assert np.array_equal(order.cpu().numpy(), rord)
    assert np.array_equal(inv.cpu().numpy(), rinv)


def _routes(rng, M, S, share=True):
    inds = np.stack([rng.choice(S, 8, replace=False) for _ in range(M)])
    if M > 1 and share:
        inds[1, :4] = inds[0, :4]
    sc = rng.random((M, 8)).astype(np.float32)
    sc /= sc.sum(1, keepdims=True)
    return inds.astype(np.int32), sc


@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_moe_experts_matches_oracle(gpu, pool24, M):
    """test_kernels.py:65-79 restated: S=24 pool, shared experts across rows."""
    import mimo_moe
    pool, opool = pool24
    rng = np.random.default_rng(10 + M)
    x = synth.hidden(M, seed=20 + M)
    inds, sc = _routes(rng, M, 24)
    g = mimo_moe.group_routes(torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu), check_rows=True)
    y = mimo_moe.moe_experts(x.to(gpu), pool, g.uids, g.urows, g.ucnt, g.uw, gather_idx=g.gather_idx,
                             num_unique=g.num_unique, pairs_rounding=(M == 1))
    xf = x.float().numpy()
    got = f32(y)
    e = O.rel_err(got, O.moe_layer(xf, opool, inds, sc))
    assert e <= TOL_ORACLE, e
    assert O.rel_err(got, O.reference_fp32(xf, opool, inds, sc)) < TOL_FP32


def test_single_expert_many_rows(gpu, pool24):
    """test_kernels.py:81-89: 8 rows x the same 4 experts, R saturated."""
    import mimo_moe
    pool, opool = pool24
    x = synth.hidden(8, seed=31)
    inds = np.tile(np.arange(4), (8, 1)).astype(np.int32)
    sc = np.full((8, 4), 0.25, np.float32)
    g = mimo_moe.group_routes(torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu), check_rows=True)
    y = mimo_moe.moe_experts(x.to(gpu), pool, g.uids, g.urows, g.ucnt, g.uw, gather_idx=g.gather_idx,
                             num_unique=g.num_unique)
    xf = x.float().numpy()
    assert O.rel_err(f32(y), O.moe_layer(xf, opool, inds, sc)) <= TOL_ORACLE
    assert O.rel_err(f32(y), O.reference_fp32(xf, opool, inds, sc)) < TOL_FP32


def test_scatter_add_path_without_gather_idx(gpu, pool24):
    import mimo_moe
    pool, opool = pool24
    rng = np.random.default_rng(5)
    x = synth.hidden(4, seed=5)
    inds, sc = _routes(rng, 4, 24)
    g = mimo_moe.group_routes(torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu))
    y = mimo_moe.moe_experts(x.to(gpu), pool, g.uids, g.urows, g.ucnt, g.uw, num_unique=g.num_unique)
    uids, urows, ucnt, uw, _ = O.group_routes(inds, sc)
    ref = O.moe_experts(x.float().numpy(), opool, uids, urows, ucnt, uw, gather_idx=None)
    assert O.rel_err(f32(y), ref) <= TOL_ORACLE


def test_negative_control_nibble_swap_is_detected(gpu, pool24):
    """A mistake planted in the oracle (nibble order swapped, the reference's own negative control)
    must make the comparison fail."""
    import mimo_moe
    pool, opool = pool24
    rng = np.random.default_rng(6)
    x = synth.hidden(2, seed=6)
    inds, sc = _routes(rng, 2, 24)
    g = mimo_moe.group_routes(torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu))
    y = f32(mimo_moe.moe_experts(x.to(gpu), pool, g.uids, g.urows, g.ucnt, g.uw, gather_idx=g.gather_idx,
                                 num_unique=g.num_unique))

    class Swapped:
        def __getitem__(self, name):
            src = synth.SynthPool(0, 0)[name]

            class T:
                def __getitem__(self, e):
                    a = src[e]
                    if name.endswith("_w"):
                        a = ((a & 0x0F0F0F0F) << 4) | ((a >> 4) & 0x0F0F0F0F)
                    return a
            return T()
    bad = O.moe_layer(x.float().numpy(), O.Pool(Swapped()), inds, sc)
    assert O.rel_err(y, bad) > 0.5


@pytest.mark.parametrize("T", [9, 64, 300])
def test_moe_prefill_matches_oracle(gpu, pool24, T):
    import mimo_moe
    pool, opool = pool24
    rng = np.random.default_rng(100 + T)
    x = synth.hidden(T, seed=40 + T)
    inds, sc = _routes(rng, T, 24, share=False)
    y = mimo_moe.moe_prefill(x.to(gpu), pool, torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu))
    assert O.rel_err(f32(y), O.moe_pairs(x.float().numpy(), opool, inds, sc)) <= TOL_ORACLE


def test_prefill_hot_expert_many_units(gpu, pool24):
    """One expert receives every token (> 64 routes -> several work units)."""
    import mimo_moe
    pool, opool = pool24
    T = 150
    x = synth.hidden(T, seed=77)
    inds = np.stack([np.r_[3, np.random.default_rng(t).choice(np.r_[0:3, 4:24], 7, replace=False)]
                     for t in range(T)]).astype(np.int32)
    sc = np.full((T, 8), 1 / 8, np.float32)
    y = mimo_moe.moe_prefill(x.to(gpu), pool, torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu))
    assert O.rel_err(f32(y), O.moe_pairs(x.float().numpy(), opool, inds, sc)) <= TOL_ORACLE


def test_prefill_through_slot_map(gpu, pool24):
    """Expert ids in [0,256) mapped onto a 24-slot pool (the reference's slot_of indirection)."""
    import mimo_moe
    pool, opool = pool24
    T = 40
    rng = np.random.default_rng(9)
    experts = rng.choice(256, 24, replace=False)
    slot_of = np.full(256, -1, np.int32)
    slot_of[experts] = np.arange(24)
    inds_slot, sc = _routes(rng, T, 24, share=False)
    inds = experts[inds_slot].astype(np.int32)
    x = synth.hidden(T, seed=8)
    y = mimo_moe.moe_prefill(x.to(gpu), pool, torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu),
                             slot_of=torch.from_numpy(slot_of).to(gpu))
    assert O.rel_err(f32(y), O.moe_pairs(x.float().numpy(), opool, inds_slot, sc)) <= TOL_ORACLE


@pytest.mark.parametrize("T", [1, 3, 9])
def test_moe_block_end_to_end(gpu, T):
    """Router + dispatch rule + experts over a full 256-expert synthetic layer; the oracle is given
    the GPU's routes (identical logits -> identical routes is checked separately)."""
    import mimo_moe
    pool = mimo_moe.ExpertPools.synthetic(256, seed=0, layer=1, device=gpu)
    opool = O.Pool(synth.SynthPool(0, 1))
    x = synth.hidden(T, seed=50 + T)
    W = synth.router_weight()
    bias = torch.zeros(256)
    y, idx, w = mimo_moe.moe_block(x.to(gpu), W.to(gpu), bias.to(gpu), pool, return_routes=True)
    idx_np, w_np = idx.cpu().numpy(), w.cpu().numpy()
    _, ri, _ = O.router(x.float().numpy(), W.float().numpy(), bias.numpy())
    # routes chosen from the GPU's logits vs the oracle's float64-rounded logits: a route flips only
    # when two selection scores sit within the logits' ~1e-6 float32 error of each other
    flipped = int(sum(len(set(a) ^ set(b)) // 2 for a, b in zip(idx_np, ri)))
    print(f"T={T}: {flipped} of {T * 8} routes differ from the oracle router's")
    assert flipped <= max(1, T * 8 // 100)
    assert O.rel_err(f32(y), O.moe_layer(x.float().numpy(), opool, idx_np, w_np)) <= TOL_ORACLE


def test_matches_reference_kernel_golden_outputs(gpu):
    """The CUDA path against outputs of the reference's own kernels A/B (tests/golden/kernels_full.npz,
    made by tests/golden/make_golden.py from engine/mimo_stream/kernels.py:33-123 run on the CPU)."""
    import mimo_moe
    from pathlib import Path
    g = np.load(Path(__file__).resolve().parent / "golden" / "kernels_full.npz")
    pool = mimo_moe.ExpertPools.synthetic(int(g["S"]), seed=int(g["seed"]), layer=int(g["layer"]), device=gpu)
    for M in g["Ms"]:
        x = torch.from_numpy(g[f"M{M}_x"].view(np.int16)).view(torch.bfloat16).to(gpu)
        inds, sc = g[f"M{M}_inds"], g[f"M{M}_scores"]
        gr = mimo_moe.group_routes(torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu), check_rows=True)
        y = mimo_moe.moe_experts(x, pool, gr.uids, gr.urows, gr.ucnt, gr.uw, gather_idx=gr.gather_idx,
                                 num_unique=gr.num_unique)
        want = O.bf16_bits_to_f32(g[f"M{M}_y"])
        assert O.rel_err(f32(y), want) <= TOL_ORACLE, M


@pytest.mark.parametrize("M", [1, 4, 8])
def test_expert_shards_reproduce_the_single_gpu_output(gpu, pool24, M):
    """Expert parallelism's arithmetic on one GPU: the per-route partials of two expert shards
    (experts 0-11 and 12-23), added and combined in route order, equal mimo_moe_experts bit for bit."""
    import mimo_moe
    pool, opool = pool24
    rng = np.random.default_rng(70 + M)
    x = synth.hidden(M, seed=80 + M)
    inds, sc = _routes(rng, M, 24)
    idx_t, w_t = torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu)
    g = mimo_moe.group_routes(idx_t, w_t, check_rows=True)
    y_ref = mimo_moe.moe_experts(x.to(gpu), pool, g.uids, g.urows, g.ucnt, g.uw, gather_idx=g.gather_idx,
                                 num_unique=g.num_unique, pairs_rounding=(M == 1))
    part = torch.zeros(M * 8, 4096, dtype=torch.float32, device=gpu)
    for lo, hi in ((0, 12), (12, 24)):
        part += mimo_moe.moe_experts_routes(x.to(gpu), pool.slice(lo, hi), idx_t, w_t, expert_base=lo,
                                            pairs_rounding=(M == 1))
    y = mimo_moe.combine(part, M, 8)
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
    assert O.rel_err(f32(y), O.moe_layer(x.float().numpy(), opool, inds, sc)) <= TOL_ORACLE


def test_routes_outside_the_shard_stay_zero(gpu, pool24):
    import mimo_moe
    pool, _ = pool24
    x = synth.hidden(2, seed=3)
    idx = torch.tensor([[0, 5, 13, 20, 1, 2, 3, 4], [23, 22, 21, 12, 6, 7, 8, 9]], dtype=torch.int32, device=gpu)
    w = torch.full((2, 8), 0.125, device=gpu)
    part = mimo_moe.moe_experts_routes(x.to(gpu), pool.slice(12, 24), idx, w, expert_base=12)
    local = ((idx >= 12) & (idx < 24)).reshape(-1)
    assert torch.all(part[~local] == 0)
    assert torch.all(part[local].abs().sum(1) > 0)


def test_negative_control_scale_off_by_one_is_detected(gpu, pool24):
    """Second planted mistake (the survey's parity rule 5): every e8m0 scale byte one too large in the
    oracle (each weight doubled) must fail the comparison."""
    import mimo_moe
    pool, _ = pool24
    rng = np.random.default_rng(16)
    x = synth.hidden(2, seed=16)
    inds, sc = _routes(rng, 2, 24)
    g = mimo_moe.group_routes(torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu))
    y = f32(mimo_moe.moe_experts(x.to(gpu), pool, g.uids, g.urows, g.ucnt, g.uw, gather_idx=g.gather_idx,
                                 num_unique=g.num_unique))

    class OffByOne:
        def __getitem__(self, name):
            src = synth.SynthPool(0, 0)[name]

            class T:
                def __getitem__(self, e):
                    a = src[e]
                    return (a + 1).astype(a.dtype) if name.endswith("_s") else a
            return T()
    bad = O.moe_layer(x.float().numpy(), O.Pool(OffByOne()), inds, sc)
    assert O.rel_err(y, bad) > 0.5


def test_downstream_logit_kl_through_a_random_head(gpu):
    """Parity reported as the mean KL of downstream logits (the real lm_head is not available): a
    seeded random bf16 head [4096 -> 32768] applied to the GPU block output and to the oracle's."""
    import mimo_moe
    pool = mimo_moe.ExpertPools.synthetic(256, seed=0, layer=2, device=gpu)
    opool = O.Pool(synth.SynthPool(0, 2))
    T = 8
    x = synth.hidden(T, seed=91)
    W = synth.router_weight()
    y, idx, w = mimo_moe.moe_block(x.to(gpu), W.to(gpu), torch.zeros(256, device=gpu), pool, return_routes=True)
    ref = O.moe_layer(x.float().numpy(), opool, idx.cpu().numpy(), w.cpu().numpy())
    g = torch.Generator().manual_seed(4)
    head = (torch.randn(4096, 32768, generator=g) * 0.02).to(torch.bfloat16).float()
    yg = y.float().cpu()
    yr = torch.from_numpy(ref).to(torch.bfloat16).float()
    lg, lr = torch.log_softmax(yg @ head * 3, -1), torch.log_softmax(yr @ head * 3, -1)
    kl = float((lr.exp() * (lr - lg)).sum(-1).mean())
    print(f"mean KL(oracle || gpu) of downstream logits: {kl:.3e}")
    assert kl < 1e-3


def test_prefill_at_full_size_agrees_with_the_per_route_path(gpu):
    """Size-independent check at BASELINE.json scale (T = 2048, 256 experts): the prefill path (64-route
    units, bf16 pair outputs, weighted fixed-order combine) against the per-route partials of the
    expert-parallel building block with bf16 rounding (the stream-K decode kernel: 8-route units, each
    512-value K group accumulated on its own and the groups added in order) followed by the route-order
    combine.  The two kernels round their float32 sums at different points, so they agree within the
    oracle bar and on nearly every bf16 output, not bit for bit."""
    import mimo_moe
    pool = mimo_moe.ExpertPools.synthetic(256, seed=0, layer=4, device=gpu)
    T = 2048
    x = synth.hidden(T, seed=77).to(gpu)
    W = synth.router_weight().to(gpu)
    idx, w = mimo_moe.router(x, W, torch.zeros(256, device=gpu))
    y_pref = mimo_moe.moe_prefill(x, pool, idx, w)
    part = mimo_moe.moe_experts_routes(x, pool, idx, w, expert_base=0, pairs_rounding=True)
    y_route = mimo_moe.combine(part, T, 8)
    same = float((y_pref.view(torch.int16) == y_route.view(torch.int16)).float().mean())
    rel = O.rel_err(f32(y_route), f32(y_pref))
    print(f"prefill vs per-route path: rel_err {rel:.2e}, identical bf16 outputs {same:.5f}")
    assert rel <= TOL_ORACLE and same >= 0.99
    # and a spot check of a few tokens against the oracle
    opool = O.Pool(synth.SynthPool(0, 4))
    rows = [0, 1000, 2047]
    ref = O.moe_pairs(x[rows].float().cpu().numpy(), opool, idx[rows].cpu().numpy(), w[rows].cpu().numpy())
    assert O.rel_err(f32(y_pref[rows]), ref) <= TOL_ORACLE


def test_combine_pairs_rows_beyond_the_grid_y_limit(gpu):
    """The weighted pair combine launches one block row per token on grid x, so an expert-parallel
    rank that receives more than 65535 routes still combines them: with one route per row, weight 1
    and the identity permutation the output equals the input bit for bit."""
    import mimo_moe
    T, H = 70001, 4096
    g = torch.Generator(device=gpu).manual_seed(11)
    yp = torch.randn(T, H, generator=g, device=gpu).to(torch.bfloat16)
    inv = torch.arange(T, dtype=torch.int32, device=gpu)
    y = mimo_moe.combine_pairs(yp, inv, torch.ones(T, 1, device=gpu), T, 1)
    assert torch.equal(y.view(torch.int16), yp.view(torch.int16))
    # two routes per token: y = bf16(fp32(a) * 0.25 + fp32(b) * 0.75), the last row included
    inv2 = torch.arange(2 * T, dtype=torch.int32, device=gpu) % T
    w2 = torch.tensor([0.25, 0.75], device=gpu).repeat(T, 1)
    y2 = mimo_moe.combine_pairs(yp, inv2, w2, T, 2)
    a, b = yp[(2 * torch.arange(T, device=gpu)) % T].float(), yp[(2 * torch.arange(T, device=gpu) + 1) % T].float()
    assert torch.equal(y2.view(torch.int16), (a * 0.25 + b * 0.75).to(torch.bfloat16).view(torch.int16))
