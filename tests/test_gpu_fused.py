"""The fused decode launch (gate/up and down in one kernel, down tiles waiting on per-unit counters)
against the two-launch path: same kernels' arithmetic, so the block output must be identical bit for
bit.  MIMO_MOE_DECODE_FUSED is read once per process, so the two-launch results come from a child
process."""
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
out = []
for T in {Ts}:
    x = synth.hidden(T, seed=70 + T).to(dev)
    y = mimo_moe.moe_block(x, W, None, pool)
    out.append(y.view(torch.int16).cpu().numpy())
np.savez({path!r}, *out)
"""


@pytest.mark.parametrize("S", [32, 256])
def test_fused_decode_equals_two_launches(gpu, tmp_path, S):
    import mimo_moe
    from oracle import synth
    Ts = [1, 2, 3, 8]
    path = str(tmp_path / "two.npz")
    env = dict(os.environ, MIMO_MOE_DECODE_FUSED="0")
    code = CHILD.format(root=str(ROOT), pkg=str(PKG_DIR), S=S, Ts=Ts, path=path)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    two = np.load(path)
    pool = mimo_moe.ExpertPools.synthetic(S, seed=0, layer=2, device=gpu)
    W = synth.router_weight(E=S).to(gpu)
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    for i, T in enumerate(Ts):
        x = synth.hidden(T, seed=70 + T).to(gpu)
        y = mimo_moe.moe_block(x, W, None, pool, status=status)
        assert np.array_equal(y.view(torch.int16).cpu().numpy(), two[f"arr_{i}"]), T
    assert int(status.item()) == 0


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
