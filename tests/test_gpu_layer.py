"""The decoder layer around the MoE block on the GPU, through the C ABI (include/mimo_moe_layer.h), against the
CPU oracle (oracle/layer_oracle.py).

Bars: RoPE + cache append within one bf16 ulp of the oracle (bit-identical on >= 99.9%); the residual add,
add + RMSNorm and SwiGLU kernels bit-identical to the oracle / to the library's separate kernels; attention
within rel_err <= 1e-2 of the float64 oracle (max |d| / max |ref|, the metric of
engine/tests/test_kernels.py:54-56; the kernel rounds P to bf16 for the P.V product) for full and sliding-window
layers, GQA groups of 16 / 8 / 1, sinks, split and unsplit key ranges, ring wrap; whole decoder layers within
1e-2 of the oracle; and the reference's decode == prefill check (engine/tests/test_parity.py:98-108) on a
two-layer stack."""
import numpy as np
import pytest
import torch

from oracle import layer_oracle as LO
from oracle import mimo_oracle as O
from oracle import synth

pytestmark = pytest.mark.gpu


def bits(t):
    return t.detach().cpu().view(torch.int16).numpy().astype(np.int32)


def f(t):
    return t.detach().float().cpu().numpy()


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def rnd(g, *shape, std=1.0):
    return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)


def _cache_from_positions(cfg, k_all, v_all, cap, gpu):
    """Cache holding positions 0..P-1 of k_all/v_all [nkv, P, d] in slots p % cap (the last `cap` survive)."""
    from mimo_moe.layer import KVCache
    c = KVCache(cfg, cap, gpu)
    P = k_all.shape[1]
    pos = torch.arange(max(0, P - cap), P)
    slots = (pos % cap).to(gpu)
    c.k[:, slots] = k_all[:, pos].to(gpu)
    c.v[:, slots] = v_all[:, pos].to(gpu)
    c.offset = P
    return c


def _cfg(kind, **kw):
    from mimo_moe.layer import mimo_full_attention, mimo_sliding_attention
    return {"full": mimo_full_attention, "swa": mimo_sliding_attention}[kind](**kw)


CASES = [
    # kind, dims overrides, T, pos0, cap, splits
    ("full", {}, 300, 0, 512, 1),
    ("full", {}, 100, 250, 512, 1),
    ("full", {}, 1, 2000, 4096, 0),
    ("full", {}, 3, 2000, 4096, 7),
    ("full", {}, 8, 2000, 4096, 1),
    ("full", {}, 8, 4000, 4096, 0),
    ("swa", {}, 300, 0, 427, 1),
    ("swa", {}, 1, 5000, 135, 0),
    ("swa", {}, 8, 5000, 135, 0),
    ("swa", {}, 8, 77, 135, 1),
    ("full", {"head_dim": 128, "v_head_dim": 128, "n_kv_heads": 8, "rotary_dim": 128}, 40, 90, 256, 0),
    # query tiles of 128 rows, no key split, cache capacity a multiple of 128: the tcgen05 kernel
    ("full", {}, 2048, 0, 2048, 1),
    ("full", {}, 37, 500, 640, 1),
    ("swa", {}, 300, 0, 512, 1),
    ("swa", {}, 200, 1000, 384, 1),
    ("full", {"head_dim": 128, "v_head_dim": 128, "n_kv_heads": 8, "rotary_dim": 128}, 40, 90, 256, 1),
    ("full", {"head_dim": 128, "v_head_dim": 128, "n_heads": 16, "n_kv_heads": 16, "rotary_dim": 128}, 300, 7, 512, 1),
    ("full", {"head_dim": 64, "v_head_dim": 64, "n_heads": 8, "n_kv_heads": 8, "rotary_dim": 32}, 5, 700, 1024, 0),
]


@pytest.mark.parametrize("kind,over,T,pos0,cap,splits", CASES)
def test_attention_matches_oracle(gpu, kind, over, T, pos0, cap, splits):
    from mimo_moe.layer import attention
    cfg = _cfg(kind, **over)
    g = torch.Generator().manual_seed(T * 7 + pos0)
    P = pos0 + T
    q = rnd(g, T, cfg.n_heads, cfg.head_dim)
    k_all = rnd(g, cfg.n_kv_heads, P, cfg.head_dim)
    v_all = rnd(g, cfg.n_kv_heads, P, cfg.v_head_dim)
    sinks = torch.randn(cfg.n_heads, generator=g) if cfg.sinks else None
    cache = _cache_from_positions(cfg, k_all, v_all, cap, gpu)
    out = attention(q.to(gpu), cache, cfg, pos0, sinks, splits=splits)
    ref = LO.attention(f(q), f(k_all), f(v_all), np.arange(pos0, P), cfg.window, cfg.scale,
                       None if sinks is None else sinks.numpy().astype(np.float64))
    got = f(out)
    assert np.isfinite(got).all()
    assert rel(got, ref) <= 1e-2
    assert np.abs(got - ref).mean() <= 3e-3 * np.abs(ref).mean()


def test_tensor_core_attention_status_stays_clear(gpu):
    """The tcgen05 kernel's bounded waits complete on an ordinary prefill call (status word still 0) and the
    output matches the split-key mma.sync kernel's on the same inputs (rel_err <= 1e-2)."""
    from mimo_moe.layer import attention
    cfg = _cfg("swa")
    g = torch.Generator().manual_seed(5)
    T, cap = 512, 768
    k_all, v_all = rnd(g, 8, T, 192), rnd(g, 8, T, 128)
    cache = _cache_from_positions(cfg, k_all, v_all, cap, gpu)
    q = rnd(g, T, 64, 192).to(gpu)
    sinks = torch.randn(64, generator=g)
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    tc = f(attention(q, cache, cfg, 0, sinks, splits=1, status=status))
    mma = f(attention(q, cache, cfg, 0, sinks, splits=2))
    assert int(status.item()) == 0
    assert rel(tc, mma) <= 1e-2


def test_attention_split_counts_agree(gpu):
    """The split count changes only the order of the float32 sums: within 1e-2 of each other."""
    from mimo_moe.layer import attention
    cfg = _cfg("full")
    g = torch.Generator().manual_seed(11)
    P = 3000
    k_all, v_all = rnd(g, 4, P, 192), rnd(g, 4, P, 128)
    cache = _cache_from_positions(cfg, k_all, v_all, 4096, gpu)
    q = rnd(g, 4, 64, 192).to(gpu)
    outs = [f(attention(q, cache, cfg, P - 4, None, splits=s)) for s in (1, 2, 5, 0)]
    for o in outs[1:]:
        assert rel(o, outs[0]) <= 1e-2


@pytest.mark.parametrize("kind,dims,T,pos0,cap", [
    # T <= 16: the warp-per-(token, head) decode kernel
    ("swa", {}, 8, 300, 135), ("full", {}, 1, 4000, 4096),
    ("swa", {"rotary_dim": 34}, 12, 0, 256),     # pass-through dims not 16-byte aligned: bf16-pair copies
    ("full", {"rotary_dim": 100}, 9, 7, 64),      # two rotary pairs per lane
    ("full", {"rotary_dim": 160}, 16, 3, 128),    # up to four rotary pairs per lane
    # larger T: one CTA per (token, 16 heads) up to 148 tokens, then CTAs walking the tokens
    ("full", {}, 37, 0, 64), ("swa", {}, 130, 10, 257), ("full", {}, 300, 5, 320),
    ("swa", {"rotary_dim": 34}, 24, 0, 256),
])
def test_rope_store_matches_oracle(gpu, kind, dims, T, pos0, cap):
    from mimo_moe.layer import KVCache, bf16_value, rope_store
    cfg = _cfg(kind, v_scale=0.707, **dims)
    g = torch.Generator().manual_seed(T)
    qkv = rnd(g, T, cfg.qkv_width)
    cache = KVCache(cfg, cap, gpu)
    q = rope_store(qkv.to(gpu), cfg, cache, pos0)
    nq, nkv, d, dv = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.v_head_dim
    x = f(qkv)
    pos = np.arange(pos0, pos0 + T)
    q_ref = LO.rope(x[:, :nq * d].reshape(T, nq, d), pos, cfg.rotary_dim, cfg.rope_theta)
    k_ref = LO.rope(x[:, nq * d:(nq + nkv) * d].reshape(T, nkv, d), pos, cfg.rotary_dim, cfg.rope_theta)
    v_ref = LO.bf16(x[:, (nq + nkv) * d:].reshape(T, nkv, dv) * bf16_value(0.707))
    slots = pos % cap
    keep = np.arange(T) >= T - cap
    qb = torch.from_numpy(q_ref).to(torch.bfloat16)
    kb = torch.from_numpy(k_ref[keep].transpose(1, 0, 2).copy()).to(torch.bfloat16)
    vb = torch.from_numpy(v_ref[keep].transpose(1, 0, 2).copy()).to(torch.bfloat16)
    dq = np.abs(bits(q) - bits(qb))
    dk = np.abs(bits(cache.k[:, slots[keep]]) - bits(kb))
    assert dq.max() <= 1 and (dq == 0).mean() >= 0.999
    assert dk.max() <= 1 and (dk == 0).mean() >= 0.999
    assert np.array_equal(bits(cache.v[:, slots[keep]]), bits(vb))


def test_residual_kernels_bit_exact(gpu):
    import mimo_moe
    from mimo_moe.layer import add, add_rmsnorm, swiglu
    g = torch.Generator().manual_seed(3)
    x, d = rnd(g, 9, 4096), rnd(g, 9, 4096, std=0.3)
    w = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)
    xg, dg, wg = x.to(gpu), d.to(gpu), w.to(gpu)
    h, r = add_rmsnorm(xg, dg, wg, 1e-5)
    h2 = add(xg, dg)
    assert torch.equal(h.view(torch.int16), h2.view(torch.int16))
    assert np.array_equal(bits(h), bits(torch.from_numpy(LO.add(f(x), f(d))).to(torch.bfloat16)))
    assert torch.equal(r.view(torch.int16), mimo_moe.rmsnorm(h2, wg, 1e-5).view(torch.int16))
    gu = rnd(g, 5, 2 * 1024, std=2.0)
    m = swiglu(gu.to(gpu))
    ref = O.swiglu_bf16(f(gu)[:, :1024], f(gu)[:, 1024:])
    assert np.array_equal(bits(m), bits(torch.from_numpy(ref).to(torch.bfloat16)))


def _oracle_attn(attn):
    c = attn.cfg
    wq, wk, wv = torch.split(attn.w_qkv, [c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim,
                                          c.n_kv_heads * c.v_head_dim])
    return LO.AttnWeights(wq=f(wq), wk=f(wk), wv=f(wv), wo=f(attn.w_o),
                          sinks=None if attn.sinks is None else f(attn.sinks).astype(np.float64),
                          n_heads=c.n_heads, n_kv_heads=c.n_kv_heads, head_dim=c.head_dim, v_head_dim=c.v_head_dim,
                          rotary_dim=c.rotary_dim, rope_theta=c.rope_theta, window=c.window, v_scale=c.v_scale)


@pytest.mark.parametrize("kind", ["full", "swa"])
def test_dense_decoder_layer_matches_oracle(gpu, kind):
    from mimo_moe.layer import DecoderLayer, synthetic_attention, synthetic_dense_mlp
    cfg = _cfg(kind, v_scale=0.707)
    attn = synthetic_attention(cfg, seed=21, device=gpu)
    mlp = synthetic_dense_mlp(inter=2048, seed=22, device=gpu)
    g = torch.Generator().manual_seed(23)
    nw = (1 + 0.1 * torch.randn(2, 4096, generator=g)).to(torch.bfloat16)
    layer = DecoderLayer(attn, mlp, nw[0], nw[1], eps=1e-5)
    cache = layer.new_cache(1024, max_chunk=160)
    a = _oracle_attn(attn)
    ocache = LO.Cache(a)
    wgu = f(mlp.w_gate_up)
    omlp = lambda r: LO.dense_mlp(r, wgu[:2048], wgu[2048:], f(mlp.w_down))  # noqa: E731
    for T in (150, 1, 8, 1):
        x = synth.hidden(T, seed=100 + T + cache.offset)
        y = f(layer(x.to(gpu), cache))
        ref = LO.decoder_layer(f(x), a, ocache, omlp, f(nw[0]), f(nw[1]), 1e-5)
        assert rel(y, ref) <= 1e-2, (T, cache.offset)
    assert cache.offset == ocache.offset == 160


def test_moe_decoder_layer_composition_and_oracle(gpu):
    """An MoE layer: the attention half against the oracle, the MoE half against the oracle's expert path on
    the GPU's routes, and the layer output = bf16(h + y) bit for bit."""
    import mimo_moe
    from mimo_moe.layer import DecoderLayer, MoEMLP, add, synthetic_attention
    S = 32
    W = synth.router_weight(E=S, seed=31).to(gpu)
    pool = mimo_moe.ExpertPools.synthetic(S, seed=0, layer=0, device=gpu)
    cfg = _cfg("swa", v_scale=0.707)
    attn = synthetic_attention(cfg, seed=32, device=gpu)
    layer = DecoderLayer(attn, MoEMLP(W, None, pool), None, None, eps=1e-6)
    seen = []
    layer.trace = lambda d: seen.append({k: v.clone() for k, v in d.items()})
    cache = layer.new_cache(512, max_chunk=64)
    a = _oracle_attn(attn)
    ocache = LO.Cache(a)
    opool = O.Pool(synth.SynthPool(0, 0), cache=16)
    for T in (40, 8, 1):
        x = synth.hidden(T, seed=200 + T).to(gpu)
        out = layer(x, cache).clone()
        s = seen[-1]
        r_ref = O.rmsnorm(f(s["x"]), None, 1e-6)
        assert np.abs(bits(s["r"]) - bits(torch.from_numpy(r_ref).to(torch.bfloat16))).max() <= 1
        a_ref = LO.attention_block(f(s["r"]), a, ocache)
        assert rel(f(s["a"]), a_ref) <= 1e-2
        y, idx, w = mimo_moe.moe_block(s["r2"], W, None, pool, return_routes=True)
        assert torch.equal(y.view(torch.int16), s["y"].view(torch.int16))
        y_ref = O.moe_layer(f(s["r2"]), opool, idx.cpu().numpy(), w.cpu().numpy())
        assert O.rel_err(f(y), y_ref) <= 1e-2
        assert torch.equal(out.view(torch.int16), add(s["h"], s["y"]).view(torch.int16))
    layer.mlp.check_status()   # no route error was recorded


def test_decode_equals_prefill_two_layers(gpu):
    """engine/tests/test_parity.py:98-108: prefill P tokens, then decode D one at a time; the decoded outputs
    match the outputs a single prefill of P + D tokens gives at those positions (max rel diff <= 1e-2)."""
    from mimo_moe.layer import DecoderLayer, synthetic_attention, synthetic_dense_mlp
    layers = []
    for i, kind in enumerate(["swa", "full"]):
        attn = synthetic_attention(_cfg(kind, v_scale=0.707), seed=40 + i, device=gpu)
        layers.append(DecoderLayer(attn, synthetic_dense_mlp(inter=2048, seed=50 + i, device=gpu), None, None))
    P, D = 200, 12
    x = synth.hidden(P + D, seed=60).to(gpu)

    def run(chunks):
        caches = [l.new_cache(512, max_chunk=P + D) for l in layers]
        outs = []
        for c0, c1 in chunks:
            h = x[c0:c1]
            for l, c in zip(layers, caches):
                h = l(h, c)
            outs.append(h)
        return torch.cat(outs)

    ref = f(run([(0, P + D)]))[P:]
    dec = f(run([(0, P)] + [(P + i, P + i + 1) for i in range(D)]))[P:]
    assert rel(dec, ref) <= 1e-2


def test_decoder_stack_matches_its_layers_and_replays_as_a_graph(gpu):
    """DecoderStack = its layers run one after another (bit for bit) over a prefill chunk and a decode step,
    and a decode step captured as a CUDA graph replays the eager step at the same position bit for bit."""
    import mimo_moe
    from mimo_moe.ep import GraphedStep
    from mimo_moe.layer import DecoderLayer, DecoderStack, MoEMLP, synthetic_attention, synthetic_dense_mlp
    S = 32
    W = synth.router_weight(E=S, seed=71).to(gpu)
    pool = mimo_moe.ExpertPools.synthetic(S, seed=0, layer=1, device=gpu)

    def build():
        return [DecoderLayer(synthetic_attention(_cfg("full", v_scale=0.707), seed=72, device=gpu),
                             synthetic_dense_mlp(inter=1024, seed=73, device=gpu), None, None),
                DecoderLayer(synthetic_attention(_cfg("swa", v_scale=0.707), seed=74, device=gpu),
                             MoEMLP(W, None, pool), None, None)]
    stack = DecoderStack(build(), max_len=512, max_chunk=64)
    ref_layers = build()
    ref_caches = [l.new_cache(512, 64) for l in ref_layers]
    for T, seed in ((50, 80), (8, 81)):
        x = synth.hidden(T, seed=seed).to(gpu)
        y = stack(x).clone()
        h = x
        for l, c in zip(ref_layers, ref_caches):
            h = l(h, c)
        assert torch.equal(y.view(torch.int16), h.view(torch.int16)), T
    pos = stack.offset
    x = synth.hidden(8, seed=82).to(gpu)
    eager = stack.at(pos)(x).clone()
    g = GraphedStep(lambda inp: stack.at(pos)(inp), 8, 4096, gpu)
    replay = g(x).clone()
    torch.cuda.synchronize()
    assert torch.equal(replay.view(torch.int16), eager.view(torch.int16))
    stack.layers[1].mlp.check_status()


@pytest.mark.parametrize("T,N,K", [(1, 13568, 4096), (8, 13568, 4096), (3, 4096, 8192), (8, 4096, 8192),
                                   (16, 1024, 256), (5, 520, 4096)])
def test_decode_linear_matches_oracle(gpu, T, N, K):
    """The decode projection kernel against the float64 oracle (nn.Linear: exact dot products rounded once
    to float32, then bf16): >= 99% of outputs identical, rel_err <= 4e-3, and outputs of at least 1% of the
    largest within two bf16 ulps (a float32 sum of thousands of products moves a near-cancelling output by an
    ulp or two; near zero an ulp count says nothing); with and without the workspace (one K segment vs the
    balanced split, summed in a fixed order); and within 1e-2 of cuBLAS."""
    from mimo_moe.layer import linear
    g = torch.Generator().manual_seed(T * 131 + N)
    x = rnd(g, T, K)
    W = rnd(g, N, K, std=0.02)
    ref = torch.from_numpy(LO.linear(f(x), f(W))).to(torch.bfloat16)
    xg, Wg = x.to(gpu), W.to(gpu)
    for ws in (True, False):
        y = linear(xg, Wg, workspace_ok=ws)
        d = np.abs(bits(y) - bits(ref))
        big = np.abs(f(ref)) >= 1e-2 * np.abs(f(ref)).max()
        assert (d == 0).mean() >= 0.99 and d[big].max() <= 2, (ws, d[big].max(), (d == 0).mean())
        assert rel(f(y), f(ref)) <= 4e-3
    assert rel(f(y), f(torch.matmul(xg, Wg.t()))) <= 1e-2
