"""Decode expert kernels (MIMO_MOE_DECODE_KERNEL, read once per process, so each variant runs in a
child process):

  e4m3        (default) two launches over whole tiles, kind::mxf8f6f4, two e4m3 activation terms; its
              down pass takes two 128-row tiles per item (MIMO_MOE_DOWN=tiles: one tile, the
              two K halves in the two accumulators, the form the one-launch kernels share);
  sk          one stream-K launch: equal K-group ranges per CTA, group partials added in a fixed
              order, kind::mxf8f6f4 with two e4m3 activation terms;
  fp4         one launch, kind::mxf4, packed weights, five e2m1 activation terms;
  e4m3-fused  the e4m3 arithmetic in one launch (down tiles wait on per-unit counters).

By default the down launch waits per unit for the gate/up launch's h (MIMO_MOE_EARLY_DOWN=0: for the
whole gate/up grid); both give the same bits.  The combine runs as its own launch by default; MIMO_MOE_DECODE_COMBINE=down runs it in the down
kernel's epilogue (with the one-tile down items), and the two must agree bit for bit.  e4m3-fused
must equal e4m3 with one-tile down items bit for bit; the paired down items sum each row's K chunks
in one accumulator instead of two halves, so they agree with it within rel_err 1e-2 and on nearly
all bf16 outputs; sk adds each 512-value K group's partial separately, so it
agrees with e4m3 within rel_err 1e-2 and on nearly all bf16 outputs; fp4 differs from them only by the activation terms' residual
(about 1e-6 of a dot product) and the sum of five accumulator columns instead of two, so its block
output stays within rel_err 1e-2 of the e4m3 path's (the oracle bar, engine/tests/test_kernels.py:54-56)
and most bf16 outputs agree exactly (the rest differ by bf16 rounding flips).  Every variant is also
held to rel_err <= 1e-2 against the CPU restatement of the reference path on the same routes."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import PKG_DIR, ROOT

pytestmark = pytest.mark.gpu

CHILD = r"""
import sys, numpy as np, torch
sys.path[:0] = [{root!r}, {pkg!r}]
import mimo_moe
from oracle import synth
dev = torch.device("cuda", 0)
pool = mimo_moe.ExpertPools.synthetic({S}, seed=0, layer=2, device=dev)
W = synth.router_weight(E={S}).to(dev)
status = torch.zeros(1, dtype=torch.int32, device=dev)
out = []
for T in {Ts}:
    x = synth.hidden(T, seed=70 + T).to(dev)
    y, idx, w = mimo_moe.moe_block(x, W, None, pool, status=status, return_routes=True)
    out += [y.view(torch.int16).cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy()]
assert int(status.item()) == 0, int(status.item())
np.savez({path!r}, *out)
"""
TS = [1, 2, 3, 8]


def _run(tmp_path, S, kernel, combine="separate", down="pairs", early="1"):
    path = str(tmp_path / f"{kernel}_{combine}_{down}_{early}_{S}.npz")
    env = dict(os.environ, MIMO_MOE_DECODE_KERNEL=kernel, MIMO_MOE_DECODE_COMBINE=combine,
               MIMO_MOE_DOWN=down, MIMO_MOE_EARLY_DOWN=early)
    code = CHILD.format(root=str(ROOT), pkg=str(PKG_DIR), S=S, Ts=TS, path=path)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    z = np.load(path)
    return [(z[f"arr_{3 * i}"], z[f"arr_{3 * i + 1}"], z[f"arr_{3 * i + 2}"]) for i in range(len(TS))]


def _oracle(gpu, S, outs):
    """The CPU restatement of the reference path (oracle/batched.py: the dispatch rule of
    engine/mimo_stream/model.py:184-219 and 324-336 over the same pool) given each run's routes."""
    import mimo_moe
    from oracle import batched as B
    from oracle import synth
    pool = B.pool_to_cpu(mimo_moe.ExpertPools.synthetic(S, seed=0, layer=2, device=gpu))
    return [B.moe_layer(synth.hidden(T, seed=70 + T).float().numpy(), pool, idx, w)
            for T, (_, idx, w) in zip(TS, outs)]


def _rel(a_bits, ref):
    a = torch.from_numpy(a_bits).view(torch.bfloat16).float().numpy()
    return float(np.abs(a - ref).max() / np.abs(ref).max())


@pytest.mark.parametrize("S", [32, 256])
def test_decode_kernels_agree(gpu, tmp_path, S):
    e4p = _run(tmp_path, S, "e4m3")                   # default: paired down items, per-unit waits
    e4w = _run(tmp_path, S, "e4m3", early="0")        # the down launch waits for the whole gate/up grid
    for (a, ia, wa), (b, ib, wb) in zip(e4p, e4w):
        assert np.array_equal(ia, ib) and np.array_equal(a, b)
    e4 = _run(tmp_path, S, "e4m3", down="tiles")
    e4s = _run(tmp_path, S, "e4m3", combine="down", down="tiles")
    for (a, ia, wa), (b, ib, wb) in zip(e4, e4s):   # combine in the down kernel == its own launch
        assert np.array_equal(ia, ib) and np.array_equal(a, b)
    for T, (a, ia, wa), (b, ib, wb), ref in zip(TS, e4, e4p, _oracle(gpu, S, e4)):
        assert np.array_equal(ia, ib)
        assert (a == b).mean() >= 0.95, (T, (a == b).mean())
        rel = _rel(b, ref)
        print(f"S={S} T={T} e4m3 paired down: rel_err vs oracle {rel:.2e}")
        assert rel <= 1e-2, (T, rel)
    e4f = _run(tmp_path, S, "e4m3-fused")
    fp4 = _run(tmp_path, S, "fp4")
    sk = _run(tmp_path, S, "sk")
    refs = _oracle(gpu, S, e4)
    for T, (a, ia, wa), (b, ib, wb), (c, ic, wc), (k, ik, wk), ref in zip(TS, e4, e4f, fp4, sk, refs):
        assert np.array_equal(ia, ib) and np.array_equal(ia, ic) and np.array_equal(wa, wc), T  # same routes
        assert np.array_equal(ia, ik) and np.array_equal(wa, wk), T
        assert np.array_equal(a, b), T
        assert (a == k).mean() >= 0.95, (T, (a == k).mean())
        for name, v in (("e4m3", a), ("fp4", c), ("sk", k)):   # each variant against the oracle itself
            rel = _rel(v, ref)
            print(f"S={S} T={T} {name}: rel_err vs oracle {rel:.2e}")
            assert rel <= 1e-2, (name, T, rel)
        fa = torch.from_numpy(a).view(torch.bfloat16).float().numpy()
        fc = torch.from_numpy(c).view(torch.bfloat16).float().numpy()
        rel = np.abs(fa - fc).max() / np.abs(fa).max()
        assert rel <= 1e-2, (T, rel)
        assert (a == c).mean() >= 0.8, (T, (a == c).mean())   # single-ulp bf16 flips only


def test_fused_decode_repeated_calls_and_graph(gpu):
    """The per-unit counters are cleared by every call: repeated eager calls and graph replays agree."""
    import mimo_moe
    from mimo_moe.ep import GraphedStep
    from oracle import synth
    pool = mimo_moe.ExpertPools.synthetic(64, seed=0, layer=4, device=gpu)
    W = synth.router_weight(E=64).to(gpu)
    xs = [synth.hidden(8, seed=s).to(gpu) for s in (1, 2, 3)]
    ref = [mimo_moe.moe_block(x, W, None, pool).clone() for x in xs]
    g = GraphedStep(lambda x: mimo_moe.moe_block(x, W, None, pool), 8, 4096, gpu)
    for rep in range(3):
        for x, r in zip(xs, ref):
            assert torch.equal(mimo_moe.moe_block(x, W, None, pool).view(torch.int16), r.view(torch.int16))
            assert torch.equal(g(x).view(torch.int16), r.view(torch.int16))


def test_back_to_back_calls_with_changing_unit_counts(gpu):
    """Launches overlap their predecessors' tails (programmatic dependent launch): a kernel must not
    read the unit count or tables before its predecessor is done.  Calls whose distinct-expert counts
    change from call to call, issued back to back, must equal the same calls run one at a time."""
    import mimo_moe
    from oracle import synth
    pool = mimo_moe.ExpertPools.synthetic(64, seed=0, layer=6, device=gpu)
    W = synth.router_weight(E=64).to(gpu)
    Ts = [8, 1, 3, 8, 2, 5, 1, 8, 4, 7]
    xs = [synth.hidden(T, seed=300 + i).to(gpu) for i, T in enumerate(Ts)]
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    fast = [mimo_moe.moe_block(x, W, None, pool, status=status) for x in xs]
    torch.cuda.synchronize()
    for x, y in zip(xs, fast):
        ref = mimo_moe.moe_block(x, W, None, pool)
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
    assert int(status.item()) == 0
