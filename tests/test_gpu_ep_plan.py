"""Expert-parallel prefill plan, row gather and receive index on the device (mimo_moe_ep_plan,
mimo_moe_gather_rows, mimo_moe_ep_recv_index) against their torch restatement (tests/ep_ref.py), bit
for bit; an exchange between simulated ranks on one GPU (every received route must see its own
token's row and its local expert id); and mimo_moe_prefill_routes against mimo_moe_prefill."""
import numpy as np
import pytest
import torch

import ep_ref

pytestmark = pytest.mark.gpu
E, K, H = 256, 8, 4096


def _idx(T, kind, seed, dev):
    g = np.random.default_rng(seed)
    if kind == "uniform":    # distinct experts per token, as the router gives
        idx = np.stack([g.choice(E, K, replace=False) for _ in range(T)])
    elif kind == "zipf":     # hot experts (config 4's skew), repeats allowed
        p = 1.0 / np.arange(1, E + 1) ** 1.1
        idx = g.choice(E, (T, K), p=p / p.sum())
    else:                    # every route to rank 0's experts
        idx = g.integers(0, 32, (T, K))
    return torch.from_numpy(idx.astype(np.int32)).to(dev)


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("T,kind", [(1, "uniform"), (7, "zipf"), (1000, "uniform"), (1025, "zipf"),
                                    (16384, "zipf"), (3000, "rank0")])
def test_plan_matches_torch(gpu, world, T, kind):
    import mimo_moe.ops as ops
    idx = _idx(T, kind, 10 * world + T, gpu)
    got = ops.ep_plan(idx, E // world, world)
    ref = ep_ref.plan(idx, E // world, world)
    torch.cuda.synchronize()
    assert torch.equal(got.counts, ref.counts)
    assert torch.equal(got.order, ref.order) and torch.equal(got.inv, ref.inv)
    rows = int(ref.counts[:, 1].sum())
    assert torch.equal(got.send_tok[:rows], ref.send_tok[:rows])
    assert torch.equal(got.send_tag, ref.send_tag)


def test_plan_reports_expert_ids_out_of_range(gpu):
    import mimo_moe.ops as ops
    from mimo_moe._lib import MIMO_ERANGE
    idx = _idx(5, "uniform", 3, gpu)
    idx[2, 4] = 300
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    p = ops.ep_plan(idx, E // 2, 2, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == MIMO_ERANGE
    assert int(p.inv[2 * K + 4]) == -1 and int(p.counts[:, 0].sum()) == 5 * K - 1


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_between_simulated_ranks(gpu, world):
    """Each simulated rank plans its own tokens; rank r receives every rank's segment for r (what the
    all-to-alls deliver) and gathers each route's row: it must be the sending token's row."""
    import mimo_moe.ops as ops
    per = E // world
    xs = [torch.randn(600 + 37 * s, H, device=gpu).to(torch.bfloat16) for s in range(world)]
    idxs = [_idx(x.shape[0], "zipf" if s % 2 else "uniform", 50 + s, gpu) for s, x in enumerate(xs)]
    plans = [ops.ep_plan(i, per, world) for i in idxs]
    sends = [ops.gather_rows(x, p.send_tok, int(p.counts[:, 1].sum())) for x, p in zip(xs, plans)]
    for x, p, sx in zip(xs, plans, sends):
        assert torch.equal(sx, ep_ref.gather_rows(x, p.send_tok, sx.shape[0]))
    for r in range(world):
        seg_rows, seg_tags, counts, origin = [], [], [], []
        for s, p in enumerate(plans):
            c = p.counts.tolist()
            r0 = sum(c[d][1] for d in range(r))
            p0 = sum(c[d][0] for d in range(r))
            seg_rows.append(sends[s][r0:r0 + c[r][1]])
            seg_tags.append(p.send_tag[p0:p0 + c[r][0]])
            counts.append(c[r])
            origin += [(s, int(q)) for q in p.order[p0:p0 + c[r][0]].tolist()]
        recv_rows, recv_tag = torch.cat(seg_rows), torch.cat(seg_tags)
        recv_counts = torch.tensor(counts, dtype=torch.int64, device=gpu)
        rr, eid = ops.ep_recv_index(recv_tag, recv_counts)
        rr_ref, eid_ref = ep_ref.recv_index(recv_tag, recv_counts)
        assert torch.equal(rr, rr_ref) and torch.equal(eid, eid_ref)
        got = recv_rows[rr.long()]
        want = torch.stack([xs[s][q // K] for s, q in origin])
        assert torch.equal(got, want)
        want_e = torch.tensor([int(idxs[s].view(-1)[q]) - r * per for s, q in origin], dtype=torch.int32,
                              device=gpu)
        assert torch.equal(eid, want_e)


def test_prefill_routes_equal_the_pair_outputs(gpu):
    """mimo_moe_prefill_routes on rows named per route gives each route's bf16 pair output: the same
    bits as mimo_moe_prefill with one route per (gathered) row and weight 1."""
    import mimo_moe
    import mimo_moe.ops as ops
    S = 32
    pool = mimo_moe.ExpertPools.synthetic(S, seed=5, layer=1, device=gpu)
    g = np.random.default_rng(9)
    rows = torch.randn(300, H, device=gpu).to(torch.bfloat16)
    P = 1000
    rr = torch.from_numpy(g.integers(0, 300, P).astype(np.int32)).to(gpu)
    e = torch.from_numpy(g.integers(0, S, P).astype(np.int32)).to(gpu)
    y = ops.moe_prefill_routes(rows, pool, rr, e)
    ref = ops.moe_prefill(rows[rr.long()], pool, e[:, None], torch.ones(P, 1, device=gpu))
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
