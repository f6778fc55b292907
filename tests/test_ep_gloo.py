"""Expert-parallel exchange logic (mimo_moe/ep.py) on CPU gloo ranks, world_size 2.

The compute steps are replaced by small deterministic CPU functions (router: top-k of x @ Wr with
normalised sigmoid weights; expert e: tanh(x @ M_e) * w; combine: float32 sum over k in order ->
bf16), so the test checks what the multi-GPU path adds: expert ownership, the all-gather dispatch,
zero partials for other ranks' experts, the exact reduce-scatter return and the fixed-order combine;
for the prefill path, the all-to-all of each route to its expert's rank (variable and empty splits),
the return and the weighted combine (with the torch restatement of the device plan, tests/ep_ref.py,
which the GPU tests hold the plan kernels to).  The EP output must equal the single-process output
bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, H, K, T = 8, 64, 3, 5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _router(x: torch.Tensor):
    wr = torch.from_numpy(np.random.default_rng(1).standard_normal((H, E)).astype(np.float32))
    s = torch.sigmoid(x.float() @ wr)
    w, idx = torch.topk(s, K, dim=1)
    return idx.to(torch.int32), (w / w.sum(1, keepdim=True)).float()


def _expert_mats():
    rng = np.random.default_rng(2)
    return [torch.from_numpy(rng.standard_normal((H, H)).astype(np.float32) / 8) for _ in range(E)]


def _experts(lo: int, hi: int):
    mats = _expert_mats()

    def fn(X, IDX, W, rnd):
        part = torch.zeros(X.shape[0] * K, H, dtype=torch.float32)
        for r in range(X.shape[0]):
            for j in range(K):
                e = int(IDX[r, j])
                if lo <= e < hi:
                    v = torch.tanh(X[r].float() @ mats[e])
                    if rnd:
                        v = v.to(torch.bfloat16).float()
                    part[r * K + j] = v * W[r, j]
        return part
    return fn


def _combine(part, M, k):
    y = torch.zeros(M, part.shape[1], dtype=torch.float32)
    for m in range(M):
        for j in range(k):
            y[m] += part[m * k + j]
    return y.to(torch.bfloat16)


def _tokens(rank: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(T, H, generator=g).to(torch.bfloat16)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mimo_moe.ep import ExpertParallelMoE, expert_range
        lo, hi = expert_range(rank, world, E)
        blk = ExpertParallelMoE(None, None, None, num_experts=E, topk=K, router_fn=_router,
                                experts_fn=_experts(lo, hi), combine_fn=_combine)
        y = blk(_tokens(rank))
        out[rank] = y.float().numpy().tobytes()
    finally:
        dist.destroy_process_group()


def test_ep_matches_single_process_bit_for_bit():
    world = 2
    port = _free_port()
    out = mp.Manager().dict()
    mp.start_processes(_worker, args=(world, port, out), nprocs=world, start_method="spawn")
    for rank in range(world):
        x = _tokens(rank)
        idx, w = _router(x)
        ref = _combine(_experts(0, E)(x, idx, w, False), T, K)
        got = np.frombuffer(out[rank], dtype=np.float32).reshape(T, H)
        assert np.array_equal(got, ref.float().numpy()), rank


def _pairs(lo: int):
    """Per-route bf16 products of the received routes (local expert ids), as the expert side of the
    all-to-all prefill computes them."""
    mats = _expert_mats()

    def fn(rows, rr, e):
        return torch.stack([torch.tanh(rows[int(rr[r])].float() @ mats[lo + int(e[r])]).to(torch.bfloat16)
                            for r in range(e.shape[0])]) if e.shape[0] else torch.empty(0, H, dtype=torch.bfloat16)
    return fn


def _combine_pairs(back, inv, w, T_, k):
    y = torch.zeros(T_, back.shape[1], dtype=torch.float32)
    for t in range(T_):
        for j in range(k):
            y[t] += back[int(inv[t * k + j])].float() * w[t, j]
    return y.to(torch.bfloat16)


def _clustered_router(x: torch.Tensor):
    """Routes that share ranks: even tokens send all K routes to rank 0's experts, odd tokens two of
    them to rank 1's (so one token row serves several routes on the receiving rank)."""
    idx, w = _router(x)
    for t in range(idx.shape[0]):
        idx[t] = torch.tensor([0, 2, 3] if t % 2 == 0 else [5, 1, 7], dtype=idx.dtype)[:K]
    return idx, w


def _prefill_worker(rank, world, port, out, clustered=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from mimo_moe.ep import ExpertParallelPrefill, expert_range
        lo, _ = expert_range(rank, world, E)
        import ep_ref
        blk = ExpertParallelPrefill(None, None, None, num_experts=E, topk=K,
                                    router_fn=_clustered_router if clustered else _router,
                                    pairs_fn=_pairs(lo), combine_fn=_combine_pairs, plan_fn=ep_ref.plan,
                                    gather_fn=ep_ref.gather_rows, recv_fn=ep_ref.recv_index)
        # rank 1 routes no tokens in the second call: empty splits both ways
        for n in (T, T if rank == 0 else 0):
            y = blk(_tokens(rank)[:n])
            assert y.shape == (n, H)
            out[(rank, n)] = y.float().numpy().tobytes()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,clustered", [(2, False), (2, True), (4, False), (4, True)])
def test_ep_prefill_all_to_all_matches_single_process(world, clustered):
    """Each token row crosses once per destination rank and serves all of its routes there (world 4:
    two experts per rank, uneven splits, ranks that send nothing to some peers)."""
    port = _free_port()
    out = mp.Manager().dict()
    mp.start_processes(_prefill_worker, args=(world, port, out, clustered), nprocs=world, start_method="spawn")
    for rank in range(world):
        x = _tokens(rank)
        idx, w = (_clustered_router if clustered else _router)(x)
        ref = _combine(_experts(0, E)(x, idx, w, True), T, K)
        got = np.frombuffer(out[(rank, T)], dtype=np.float32).reshape(T, H)
        assert np.array_equal(got, ref.float().numpy()), rank
    assert out[(1, 0)] == b""


def test_expert_ranges_and_rounding_rule():
    from mimo_moe.ep import expert_range, pairs_rounding_for
    assert [expert_range(r, 8) for r in (0, 7)] == [(0, 32), (224, 256)]
    with pytest.raises(ValueError):
        expert_range(0, 3)
    assert [pairs_rounding_for(t) for t in (1, 2, 8, 9, 2048)] == [True, False, False, True, True]
