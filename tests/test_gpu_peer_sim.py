"""The expert-parallel decode exchange's kernels on ONE GPU, with two simulated ranks.

The multi-GPU exchange (mimo_moe.ep.PeerExpertParallelMoE) routes each rank's tokens and stores every
token's packed row [x | ids | weights] into every rank's gather buffer (route_scatter_kernel), builds
the local experts' work units from all ranks' routes (routes_prep_kernel), and stores each route's
float32 partial straight into the owner rank's receive buffer from the down kernel's epilogue, before
the owner's fixed-order combine.  Here both ranks' buffers live on one device and the ranks' steps run
one after the other on one stream (so no flag barrier is needed: stream order already puts every
scatter before every expert pass, and every expert pass before every combine).  Each simulated rank's
output must equal the single-GPU block on its own tokens bit for bit: the reference computes the layer
on one device (engine/mimo_stream/model.py:303-336, kernels.py:176-199), and every route's partial is
the same arithmetic whatever rank computes it.

Also: a barrier wait that nothing completes expires after its limit and reports MIMO_ETIMEOUT instead
of hanging (the reference surfaces I/O and routing failures as errors, never as a hang:
engine/mimo_stream/store.py:55-57, kernels.py:167-168)."""
import time

import numpy as np
import pytest
import torch

from oracle import synth

pytestmark = pytest.mark.gpu

E, K, H, I = 256, 8, 4096, 2048


@pytest.fixture(scope="module")
def layer(gpu):
    import mimo_moe
    pool = mimo_moe.ExpertPools.synthetic(E, seed=0, layer=5, device=gpu)
    torch.cuda.synchronize()
    return pool, synth.router_weight().to(gpu)


@pytest.mark.parametrize("N,T", [(2, 1), (2, 8), (4, 3)])
def test_peer_exchange_kernels_with_simulated_ranks_equal_the_single_gpu_block(gpu, layer, N, T):
    import mimo_moe
    from mimo_moe import _lib
    from mimo_moe.ep import expert_range, pairs_rounding_for
    L = mimo_moe.lib()
    pool, W = layer
    ld = H // 2 + 2 * K
    per = E // N
    st = torch.cuda.current_stream().cuda_stream
    rows = [torch.zeros(N * T, ld, dtype=torch.int32, device=gpu) for _ in range(N)]
    recv = [torch.full((T * K, H), float("nan"), dtype=torch.float32, device=gpu) for _ in range(N)]
    rows_tab = torch.tensor([r.data_ptr() for r in rows], dtype=torch.int64, device=gpu)
    recv_tab = torch.tensor([r.data_ptr() for r in recv], dtype=torch.int64, device=gpu)
    xs = [synth.hidden(T, seed=500 + 10 * T + r).to(gpu) for r in range(N)]
    logits = [torch.empty(T, E, dtype=torch.float32, device=gpu) for _ in range(N)]
    ys = [torch.empty(T, H, dtype=torch.bfloat16, device=gpu) for _ in range(N)]
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    nb = L.mimo_moe_experts_routes_workspace_bytes(N * T, K, H, I, per)
    ws = [torch.empty(nb, dtype=torch.uint8, device=gpu) for _ in range(N)]
    for r in range(N):      # every rank's dispatch lands in every rank's gather buffer
        _lib.check(L.mimo_moe_route_scatter(xs[r].data_ptr(), T, H, W.data_ptr(), None, E, K, rows_tab.data_ptr(),
                                            ld, r, N, logits[r].data_ptr(), st), "route_scatter")
    for r in range(N):      # each rank's experts over all ranks' tokens; partials into the owners' buffers
        lo, hi = expert_range(r, N, E)
        shard = pool.slice(lo, hi)
        base = rows[r].data_ptr()
        _lib.check(L.mimo_moe_experts_routes(base, 2 * ld, N * T, shard.struct, lo, base + 2 * H, base + 2 * H + 4 * K,
                                             ld, K, int(pairs_rounding_for(T)), None, recv_tab.data_ptr(), T * K,
                                             ws[r].data_ptr(), ws[r].numel(), status.data_ptr(), st),
                   "experts_routes")
    for r in range(N):
        _lib.check(L.mimo_moe_combine(recv[r].data_ptr(), T * K, None, T, K, H, ys[r].data_ptr(), status.data_ptr(),
                                      st), "combine")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for r in range(1, N):
        assert torch.equal(rows[r], rows[0])  # identical gather buffers on every rank
    for r in range(N):
        assert torch.isfinite(recv[r]).all()  # every route's partial was stored exactly once, by its expert's rank
        want = mimo_moe.moe_block(xs[r], W, None, pool)
        assert torch.equal(ys[r].view(torch.int16), want.view(torch.int16)), r


def test_barrier_wait_that_never_completes_expires_with_a_timeout(gpu):
    """Rank 0 of two waits for a rank 1 that never arrives: the wait gives up after its 20 ms limit,
    MIMO_ETIMEOUT lands in the status word, and the context stays usable (a second barrier whose peer
    signal is already there passes)."""
    import mimo_moe
    from mimo_moe import _lib
    L = mimo_moe.lib()
    st = torch.cuda.current_stream().cuda_stream
    sig = [torch.zeros(64, dtype=torch.int32, device=gpu) for _ in range(2)]  # rank 0's and rank 1's signal arrays
    tab = torch.tensor([s.data_ptr() for s in sig], dtype=torch.int64, device=gpu)
    epoch = torch.zeros(1, dtype=torch.int32, device=gpu)
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(L.mimo_moe_peer_barrier(tab.data_ptr(), sig[0].data_ptr(), 0, 2, epoch.data_ptr(), 20000,
                                       status.data_ptr(), st), "peer_barrier")
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(status.item()) == _lib.MIMO_ETIMEOUT
    assert dt < 1.5, dt                          # the 20 ms limit, not the 2 s default
    assert int(sig[1][0].item()) == 1            # rank 0 did signal rank 1's slot 0
    assert int(epoch.item()) == 1
    # the peer's signal for the next epoch is already there: no wait, no error
    sig[0][1] = 2
    status.zero_()
    _lib.check(L.mimo_moe_peer_barrier(tab.data_ptr(), sig[0].data_ptr(), 0, 2, epoch.data_ptr(), 20000,
                                       status.data_ptr(), st), "peer_barrier")
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and int(epoch.item()) == 2
    x = torch.ones(4, device=gpu)
    assert float((x * 2).sum().item()) == 8.0
