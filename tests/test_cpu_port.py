"""The native CPU baseline kernel (oracle/cpu_mxfp4.c: the reference's kernels A/B over the packed MXFP4 bytes,
timed as the fastest CPU form of the path) against a float64 restatement of the same expert on the same rows,
and its AVX2 path bit-identical to its scalar path.  Test infrastructure checking test infrastructure: the
timed baseline must compute the path it claims to time."""
import numpy as np
import pytest
import torch

from oracle import batched as B
from oracle import cpu_path
from oracle import mimo_oracle as O
from oracle import synth


@pytest.fixture(scope="module")
def lib():
    from oracle import cpu_port_build
    cpu_port_build.build()
    L = cpu_path.native()
    assert L is not None
    return L


def _expert(e):
    sp = synth.SynthPool(0, 0)
    return {n: torch.from_numpy(np.ascontiguousarray(sp[n][e]).view(np.int32 if n.endswith("_w") else np.uint8))
            for n in ("gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")}


def _reference(raw, X, pairs):
    """float64 products of the dequantised weights with the kernels' roundings (bf16 g, u, SwiGLU)."""
    Wg, Wu, Wd = (B.dequant(raw[f"{n}_w"], raw[f"{n}_s"]).double() for n in ("gate", "up", "down"))
    x = X.double()
    g = (x @ Wg.T).float().numpy()
    u = (x @ Wu.T).float().numpy()
    h = O.swiglu_bf16(g, u)
    d = (torch.from_numpy(np.asarray(h, np.float64)) @ Wd.T).float().numpy()
    return h, (O.bf16_round(d) if pairs else d)


@pytest.mark.parametrize("e,R,pairs", [(3, 1, True), (77, 3, False), (200, 8, False), (5, 11, True)])
def test_native_expert_matches_the_float64_restatement(lib, e, R, pairs):
    raw = _expert(e)
    X = synth.hidden(R, seed=40 + R)
    got = cpu_path.native_expert(raw, X, pairs).numpy()
    _, want = _reference(raw, X, pairs)
    assert O.rel_err(got, want) <= 1e-2
    assert np.mean(O.bf16_round(got) == O.bf16_round(want)) >= 0.9


def test_avx2_and_scalar_paths_agree_bit_for_bit(lib):
    if lib.mimo_cpu_port_isa() != 2:
        pytest.skip("host without AVX2 + FMA: only the scalar path exists")
    raw = _expert(9)
    X = synth.hidden(5, seed=3)
    fast = cpu_path.native_expert(raw, X, False).numpy()
    lib.mimo_cpu_port_force_scalar(1)
    try:
        slow = cpu_path.native_expert(raw, X, False).numpy()
    finally:
        lib.mimo_cpu_port_force_scalar(0)
    assert np.array_equal(fast.view(np.uint32), slow.view(np.uint32))


class _LazyPool:
    """pool[key][expert] -> that expert's tensor, generated on demand (the batched oracle's pool access)."""

    def __init__(self, get):
        self.get = get

    def __getitem__(self, key):
        get = self.get

        class _Proj:
            def __getitem__(self, e):
                return get(int(e))[key]
        return _Proj()


@pytest.mark.parametrize("T,cached,packed", [(1, True, False), (3, True, False), (1, False, False),
                                             (1, False, True), (3, False, True)])
def test_timed_cpu_layer_computes_the_moe_layer(lib, T, cached, packed):
    """The timed CPU step itself (router, every distinct expert, the fixed-order combine) against the batched
    oracle on the same routes (the reference's dispatch rule: pair path at T = 1, kernels A/B at 2..8)."""
    cache = {}

    def get(e):
        if e not in cache:
            cache[e] = _expert(e)
        return cache[e]
    W = synth.router_weight()
    layer = cpu_path.CpuLayer(W, torch.zeros(W.shape[0]), get)
    x = synth.hidden(T, seed=60 + T)
    outs = []
    _, done, U = layer.step_time(x, cached, budget_s=1e9, packed=packed, outputs=outs)
    assert done == U
    y, inds, w = outs[0]
    want = B.moe_layer(x.float().numpy(), _LazyPool(get), inds.numpy(), w.numpy())
    assert O.rel_err(y.numpy(), want) <= 1e-2
