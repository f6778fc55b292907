"""RMSNorm and the multi-layer decode stack on the GPU, through the C ABI.

Bars: RMSNorm within one bf16 ulp of the oracle everywhere and bit-identical on >= 99.9% of elements
(the oracle's float64 sum of squares versus the kernel's fixed float32 order); the stack equals the
layer-by-layer composition of the library's own ops bit for bit, eager and replayed as a CUDA graph;
each layer of a stack run matches the oracle's MoE block on that layer's input (rel_err <= 1e-2, the
metric of engine/tests/test_kernels.py:54-56) and the oracle's RMSNorm of the previous layer's output."""
import numpy as np
import pytest
import torch

from oracle import mimo_oracle as O
from oracle import synth

pytestmark = pytest.mark.gpu

S = 32  # experts per layer in these tests (the smallest pool the block accepts)


def bits(t):
    return t.detach().cpu().view(torch.int16).numpy().astype(np.int32)


def ulp_diff(a, b):
    """Distance in bf16 ulps between two bf16 tensors of the same sign pattern."""
    return np.abs(bits(a) - bits(b))


@pytest.mark.parametrize("T,scale", [(1, 1.0), (37, 1.0), (5, 1e-3), (8, 300.0), (70001, 1.0)])
def test_rmsnorm_matches_oracle(gpu, T, scale):
    import mimo_moe
    g = torch.Generator().manual_seed(T)
    x = (torch.randn(T, 4096, generator=g) * scale).to(torch.bfloat16)
    y = mimo_moe.rmsnorm(x.to(gpu))
    ref = torch.from_numpy(O.rmsnorm(x.float().numpy())).to(torch.bfloat16)
    d = ulp_diff(y, ref)
    assert d.max() <= 1 and (d == 0).mean() >= 0.999


def test_rmsnorm_weight_and_in_place(gpu):
    import mimo_moe
    g = torch.Generator().manual_seed(5)
    x = torch.randn(9, 4096, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    y = mimo_moe.rmsnorm(x.to(gpu), w.to(gpu))
    ref = torch.from_numpy(O.rmsnorm(x.float().numpy(), w.float().numpy())).to(torch.bfloat16)
    d = ulp_diff(y, ref)
    assert d.max() <= 1 and (d == 0).mean() >= 0.999
    xd = x.to(gpu)
    y0 = mimo_moe.rmsnorm(xd)
    mimo_moe.rmsnorm(xd, out=xd)                 # x == y is allowed
    assert torch.equal(xd.view(torch.int16), y0.view(torch.int16))


def test_rmsnorm_rejects_bad_shapes(gpu):
    import mimo_moe
    with pytest.raises(ValueError):          # MIMO_EINVAL, raised as the reference raises shape errors
        mimo_moe.rmsnorm(torch.zeros(2, 12, dtype=torch.bfloat16, device=gpu))


def _layers(gpu, L):
    import mimo_moe
    out = []
    for l in range(L):
        W = synth.router_weight(E=S, seed=1 + 1000 * l)
        pool = mimo_moe.ExpertPools.synthetic(S, seed=0, layer=l, device=gpu)
        out.append((W.to(gpu), None, pool))
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("T", [1, 8, 20])
def test_stack_equals_layerwise_composition_eager_and_graphed(gpu, T):
    import mimo_moe
    from mimo_moe.ep import GraphedStep
    layers = _layers(gpu, 3)
    stack = mimo_moe.MoEStack(layers)
    x = synth.hidden(T, seed=40 + T).to(gpu)
    want = x
    for l, (W, b, pool) in enumerate(layers):
        if l:
            want = mimo_moe.rmsnorm(want)
        want = mimo_moe.moe_block(want, W, b, pool)
    got = stack(x).clone()
    g = GraphedStep(stack, T, 4096, gpu)
    replay = [g(synth.hidden(T, seed=s).to(gpu)).clone() for s in (7, 40 + T)]
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert torch.equal(replay[1].view(torch.int16), want.view(torch.int16))
    assert not torch.equal(replay[0].view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("T", [1, 2])
def test_stack_layers_against_oracle(gpu, T):
    import mimo_moe
    layers = _layers(gpu, 2)
    stack = mimo_moe.MoEStack(layers)
    seen = []
    stack.on_layer = lambda l, x: seen.append(x.clone())
    y_last = stack(synth.hidden(T, seed=90 + T).to(gpu)).clone()
    torch.cuda.synchronize()
    assert len(seen) == 2
    for l, (W, _, pool) in enumerate(layers):
        x_l = seen[l]
        y_l, idx, w = mimo_moe.moe_block(x_l, W, None, pool, return_routes=True)
        if l == 1:
            assert torch.equal(y_l.view(torch.int16), y_last.view(torch.int16))
        xf = x_l.float().cpu().numpy()
        _, ri, _ = O.router(xf, W.float().cpu().numpy(), np.zeros(S, np.float32))
        assert (np.sort(idx.cpu().numpy(), 1) == np.sort(ri, 1)).mean() > 0.99
        opool = O.Pool(synth.SynthPool(0, l), cache=16)
        ref = O.moe_layer(xf, opool, idx.cpu().numpy(), w.cpu().numpy())
        assert O.rel_err(y_l.float().cpu().numpy(), ref) <= 1e-2, l
        if l == 0:   # the next layer's input is the oracle's RMSNorm of this output
            d = ulp_diff(seen[1], torch.from_numpy(O.rmsnorm(y_l.float().cpu().numpy())).to(torch.bfloat16))
            assert d.max() <= 1
