"""Parity at the BASELINE.json sizes (full 256-expert MiMo layer), through the C ABI, against the batched CPU
restatement of the reference's pair path (oracle/batched.py, pinned bit for bit to oracle/mimo_oracle.py
by tests/test_oracle.py).

  config 2  prefill of 2048 tokens, free routing: every output row, so every expert, every 64-route work
            unit and every unit boundary is covered;
  config 4  prefill of 16384 tokens with the Zipf(1.1)-biased router (hottest experts ~10x the mean
            load, i.e. dozens of 64-route units each): the rows of the five hottest experts at each of
            their unit boundaries, plus a seeded sample of other rows.

The oracle is given the GPU's routes (the router itself is checked bit for bit against the oracle given
identical logits in test_gpu_parity.py).  Bar: rel_err = max|a - b| / max|b| <= 1e-2 (engine/tests/
test_kernels.py:54-56, the metric of the reference's own kernel tests), on the whole output and per row;
the share of bit-identical bf16 outputs is reported."""
import numpy as np
import pytest
import torch

from oracle import batched as B
from oracle import mimo_oracle as O
from oracle import synth

pytestmark = pytest.mark.gpu

TOL = 1e-2
UNIT = 64  # routes per prefill work unit of the tensor-core kernels


@pytest.fixture(scope="module")
def layer(gpu):
    import mimo_moe
    pool = mimo_moe.ExpertPools.synthetic(256, seed=0, layer=4, device=gpu)
    torch.cuda.synchronize()
    return pool, B.pool_to_cpu(pool)


def _check(y, ref, what):
    got = y.float().cpu().numpy()
    e = O.rel_err(got, ref)
    per_row = np.abs(got - ref).max(1) / (np.abs(ref).max(1) + 1e-9)
    same = (O.f32_to_bf16_bits(got) == O.f32_to_bf16_bits(ref)).mean()
    print(f"{what}: rel_err {e:.2e}, worst row {per_row.max():.2e}, identical bf16 outputs {same:.4f}")
    assert e <= TOL, e
    assert per_row.max() <= 2 * TOL, per_row.max()
    return same


def test_prefill2048_every_row_matches_the_oracle(gpu, layer):
    import mimo_moe
    pool, cpool = layer
    T = 2048
    x = synth.hidden(T, seed=77)
    W = synth.router_weight()
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    y, idx, w = mimo_moe.moe_block(x.to(gpu), W.to(gpu), torch.zeros(256, device=gpu), pool, status=status,
                                   return_routes=True)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    inds = idx.cpu().numpy()
    counts = np.bincount(inds.reshape(-1), minlength=256)
    assert (counts > 0).all() and (counts > UNIT).any()  # every expert, and multi-unit experts, covered
    ref = B.moe_pairs(x.float().numpy(), cpool, inds, w.cpu().numpy())
    _check(y, ref, "prefill2048, all rows")


def test_prefill16384_zipf_hot_experts_match_the_oracle(gpu, layer):
    import mimo_moe
    pool, cpool = layer
    T = 16384
    x = synth.hidden(T, seed=2)
    W = synth.router_weight()
    bias = synth.zipf_bias(c=0.055)
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    y, idx, w = mimo_moe.moe_block(x.to(gpu), W.to(gpu), bias.to(gpu), pool, status=status, return_routes=True)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    inds = idx.cpu().numpy()
    flat = inds.reshape(-1)
    counts = np.bincount(flat, minlength=256)
    hot = np.argsort(-counts, kind="stable")[:5]
    assert counts[hot[0]] >= 8 * counts.mean()          # the skew the config asks for (~10x the mean)
    rows = set()
    for e in hot:  # dispatch keeps routes in (token, k) order within an expert: unit u = routes [64u, 64u+64)
        toks = np.nonzero(flat == e)[0] // inds.shape[1]
        for u0 in range(0, len(toks), UNIT):
            rows.update(int(toks[i]) for i in (u0, min(u0 + UNIT, len(toks)) - 1))
    rng = np.random.default_rng(5)
    rows.update(int(r) for r in rng.choice(T, 64, replace=False))
    rows = np.array(sorted(rows))
    units = sum((counts[e] + UNIT - 1) // UNIT for e in hot)
    print(f"config 4: hottest loads {counts[hot].tolist()} (mean {counts.mean():.0f}), {units} units, "
          f"{len(rows)} rows checked")
    ref = B.moe_pairs(x[rows].float().numpy(), cpool, inds[rows], w.cpu().numpy()[rows])
    _check(y[torch.from_numpy(rows).to(gpu)], ref, "prefill16384 Zipf, hot-expert unit boundaries")
