"""Bad route tables are reported, not followed out of bounds.

The reference raises ValueError when more than R rows are routed to one expert (engine/mimo_stream/
kernels.py:167-168); the C ABI reports such tables, and any index outside the buffers it was given,
as MIMO_ERANGE in the status word, and its kernels then clamp the index instead of following it.
Each case here hands mimo_moe_experts (or the static-scratch entry) one bad table, checks the code,
and checks that nothing past the caller's buffers was written: the workspace is followed by a guard
region inside the same allocation."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import synth

pytestmark = pytest.mark.gpu

GUARD = 1 << 20
ERANGE = 2


@pytest.fixture(scope="module")
def pool8(gpu):
    import mimo_moe
    p = mimo_moe.ExpertPools.synthetic(8, seed=0, layer=7, device=gpu)
    torch.cuda.synchronize()
    return p


def _tables(gpu, ucnt, R, urows=None, uslot=None):
    U = len(ucnt)
    urows = torch.zeros(U, R, dtype=torch.int32) if urows is None else torch.tensor(urows, dtype=torch.int32)
    uw = torch.full((U, R), 0.125, dtype=torch.float32)
    uslot = torch.arange(U, dtype=torch.int32) if uslot is None else torch.tensor(uslot, dtype=torch.int32)
    return [t.contiguous().to(gpu) for t in (uslot, urows, torch.tensor(ucnt, dtype=torch.int32), uw)]


def _experts(gpu, pool, M, tables, R, gidx=None, topk=8):
    """mimo_moe_experts through the C ABI with a guard region after the workspace."""
    import mimo_moe
    L = mimo_moe.lib()
    uslot, urows, ucnt, uw = tables
    U = uslot.numel()
    nb = L.mimo_moe_experts_workspace_bytes(M, U, R, 4096, 2048)
    buf = torch.full((nb + GUARD,), 0xA5, dtype=torch.uint8, device=gpu)
    x = synth.hidden(M, seed=4).to(gpu)
    y = torch.empty(M, 4096, dtype=torch.bfloat16, device=gpu)
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    rc = L.mimo_moe_experts(x.data_ptr(), ctypes.byref(pool.struct), uslot.data_ptr(), urows.data_ptr(),
                            ucnt.data_ptr(), uw.data_ptr(), None, U, R, None if gidx is None else gidx.data_ptr(),
                            topk, M, 0, y.data_ptr(), buf.data_ptr(), nb, status.data_ptr(),
                            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0
    assert torch.all(buf[nb:] == 0xA5), "write past the workspace"
    return int(status.item()), y


def test_more_routes_than_R_on_one_unit_is_reported_and_contained(gpu, pool8):
    # R = 4 route slots per unit, the last unit claims 8: its routes 4..7 would land past part's U*R rows
    st, y = _experts(gpu, pool8, 2, _tables(gpu, [2, 8], R=4, urows=[[0, 1, 0, 0], [0, 1, 1, 0]]), R=4)
    assert st == ERANGE
    assert torch.isfinite(y.float()).all()


def test_gather_idx_beyond_the_partials_is_reported_and_skipped(gpu, pool8):
    tables = _tables(gpu, [1, 1], R=8, urows=[[0] * 8, [0] * 8])
    gidx = torch.tensor([0, 8, 5000, -1], dtype=torch.int32, device=gpu)   # 5000 >= U * R = 16
    st, y = _experts(gpu, pool8, 1, tables, R=8, gidx=gidx, topk=4)
    assert st == ERANGE
    assert torch.isfinite(y.float()).all()
    # the same call with the bad entry dropped gives the same output: it was skipped, not read
    st2, y2 = _experts(gpu, pool8, 1, tables, R=8, gidx=torch.tensor([0, 8, -1, -1], dtype=torch.int32, device=gpu),
                       topk=4)
    assert st2 == 0 and torch.equal(y.view(torch.int16), y2.view(torch.int16))


def test_route_row_beyond_the_batch_is_reported(gpu, pool8):
    # M = 2 token rows; a route names row 6
    st, y = _experts(gpu, pool8, 2, _tables(gpu, [2], R=8, urows=[[0, 6, 0, 0, 0, 0, 0, 0]]), R=8)
    assert st == ERANGE


def test_static_entry_reports_bad_tables(gpu, pool8):
    import mimo_moe
    L = mimo_moe.lib()
    for ucnt, urows in (([2, 8], [[0, 1, 0, 0], [0, 1, 1, 0]]), ([2, 1], [[0, 5, 0, 0], [1, 0, 0, 0]])):
        uslot, urows_t, ucnt_t, uw = _tables(gpu, ucnt, R=4, urows=urows)
        x = synth.hidden(2, seed=4).to(gpu)
        y = torch.empty(2, 4096, dtype=torch.bfloat16, device=gpu)
        status = torch.zeros(1, dtype=torch.int32, device=gpu)
        rc = L.mimo_moe_experts_static(x.data_ptr(), ctypes.byref(pool8.struct), uslot.data_ptr(), urows_t.data_ptr(),
                                       ucnt_t.data_ptr(), uw.data_ptr(), None, 2, 4, None, 8, 2, 0, y.data_ptr(),
                                       status.data_ptr(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert rc == 0 and int(status.item()) == ERANGE


def test_combine_reports_rows_beyond_part(gpu):
    import mimo_moe
    L = mimo_moe.lib()
    part = torch.randn(16, 4096, device=gpu)
    y = torch.empty(2, 4096, dtype=torch.bfloat16, device=gpu)
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    gidx = torch.tensor([0, 1, 2, 99, 4, 5, 6, 7], dtype=torch.int32, device=gpu)
    rc = L.mimo_moe_combine(part.data_ptr(), 16, gidx.data_ptr(), 2, 4, 4096, y.data_ptr(), status.data_ptr(),
                            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0 and int(status.item()) == ERANGE
    want = (part[0] + part[1] + part[2]).to(torch.bfloat16)
    assert torch.equal(y[0].view(torch.int16), want.view(torch.int16))
