"""mimo_moe_experts_static: the expert products for callers that cannot allocate device memory.

Such callers (a runtime that hands the library only activations and weights, code confined to a fixed
preallocated arena, a process barred from cudaMalloc) use the entry point whose scratch is a fixed
device array inside the library.  Here it is called through the C ABI several times in a row on
different routes, and each result is compared with the workspace-taking entry point mimo_moe_experts
and with the CPU restatement of the reference path (oracle/batched.py, the kernels A/B arithmetic of
engine/mimo_stream/kernels.py:33-123 and the combine of :194-199), including a call without
gather_idx (the scatter-add order of kernels.py:196-197) and one with R = 4 route slots per expert."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import batched as B
from oracle import mimo_oracle as O
from oracle import synth

pytestmark = pytest.mark.gpu

TOL = 1e-2  # the output tolerance of the other GPU parity tests


def _routes(rng, M, S):
    inds = np.stack([rng.choice(S, 8, replace=False) for _ in range(M)]).astype(np.int32)
    if M > 1:
        inds[1, :4] = inds[0, :4]
    sc = rng.random((M, 8)).astype(np.float32)
    return inds, sc / sc.sum(1, keepdims=True)


def test_static_scratch_entry_matches_workspace_entry(gpu):
    import mimo_moe
    L = mimo_moe.lib()
    pool = mimo_moe.ExpertPools.synthetic(32, seed=3, layer=2, device=gpu)
    cpool = B.pool_to_cpu(pool)
    assert L.mimo_moe_experts_static_scratch_bytes() >= 8 * 4096 * 2 + 512 * (2048 * 2 + 4096 * 4)
    rng = np.random.default_rng(42)
    stream = torch.cuda.current_stream().cuda_stream
    # calls in a row: (rows, route slots per expert, gather_idx given)
    for call, (M, R, with_gidx) in enumerate(((8, 8, True), (3, 8, True), (3, 4, False), (8, 8, True))):
        x = synth.hidden(M, seed=900 + call).to(gpu)
        inds, sc = _routes(rng, M, 32)
        g = mimo_moe.group_routes(torch.from_numpy(inds).to(gpu), torch.from_numpy(sc).to(gpu), R=R,
                                  check_rows=True)
        gi = g.gather_idx if with_gidx else None
        want = mimo_moe.moe_experts(x, pool, g.uids, g.urows, g.ucnt, g.uw, R=R, gather_idx=gi,
                                    num_unique=g.num_unique)
        y = torch.empty(M, 4096, dtype=torch.bfloat16, device=gpu)
        status = torch.zeros(1, dtype=torch.int32, device=gpu)
        rc = L.mimo_moe_experts_static(x.data_ptr(), ctypes.byref(pool.struct), g.uids.data_ptr(),
                                       g.urows.data_ptr(), g.ucnt.data_ptr(), g.uw.data_ptr(),
                                       g.num_unique.data_ptr(), g.uids.numel(), R,
                                       gi.data_ptr() if gi is not None else None,
                                       8, M, 0, y.data_ptr(), status.data_ptr(), stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        got = y.float().cpu().numpy()
        assert O.rel_err(got, want.float().cpu().numpy()) <= TOL, call
        ref = B.moe_grouped(x.float().cpu().numpy(), cpool, inds, sc, unit_order=not with_gidx)
        assert O.rel_err(got, ref) <= TOL, call


def test_static_scratch_entry_refuses_oversized_calls(gpu):
    import mimo_moe
    L = mimo_moe.lib()
    pool = mimo_moe.ExpertPools.synthetic(32, seed=3, layer=2, device=gpu)
    dummy = torch.zeros(16, dtype=torch.int32, device=gpu)
    p = dummy.data_ptr()
    ERANGE = 2
    # M = 9 rows exceeds the fixed scratch; nothing is launched
    assert L.mimo_moe_experts_static(p, ctypes.byref(pool.struct), p, p, p, p, None, 8, 8, p, 8, 9, 0, p,
                                     None, None) == ERANGE
    # U*R = 65*8 route slots exceeds it too
    assert L.mimo_moe_experts_static(p, ctypes.byref(pool.struct), p, p, p, p, None, 65, 8, p, 8, 8, 0, p,
                                     None, None) == ERANGE
