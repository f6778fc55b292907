"""CPU checks of the decoder-layer oracle (oracle/layer_oracle.py) and of the layer C ABI's host-side argument
checks (no GPU): RoPE against the pairwise rotation it restates, the sink as an extra softmax logit, the
sliding-window mask against a brute-force loop, and decode == prefill inside the oracle (the reference's own
check of the two paths, engine/tests/test_parity.py:98-108)."""
import numpy as np
import pytest

from oracle import layer_oracle as LO
from oracle.mimo_oracle import bf16_round


def _bf(rng, *shape, std=1.0):
    return bf16_round((rng.standard_normal(shape) * std).astype(np.float32))


def test_rope_rotates_pairs_and_leaves_the_other_dims():
    rng = np.random.default_rng(0)
    x = _bf(rng, 3, 2, 16)
    pos = np.array([0, 5, 1000])
    y = LO.rope(x, pos, 8, 10000.0)
    assert np.array_equal(y[0], x[0])                   # position 0: identity
    assert np.array_equal(y[..., 8:], x[..., 8:])       # dims beyond rotary_dim pass through
    for t, p in enumerate(pos):
        for i in range(4):
            a = p * 10000.0 ** (-2 * i / 8)
            z = complex(float(x[t, 1, i]), float(x[t, 1, i + 4])) * complex(np.cos(a), np.sin(a))
            assert abs(float(y[t, 1, i]) - z.real) <= 2 ** -7 * max(1.0, abs(z.real))
            assert abs(float(y[t, 1, i + 4]) - z.imag) <= 2 ** -7 * max(1.0, abs(z.imag))


def test_sink_is_one_more_logit_without_a_value():
    rng = np.random.default_rng(1)
    T, nq, nkv, d, P = 3, 4, 2, 16, 7
    q, k, v = _bf(rng, T, nq, d), _bf(rng, nkv, P, d), _bf(rng, nkv, P, d)
    qpos = np.array([4, 5, 6])
    plain = LO.attention(q, k, v, qpos, 0, d ** -0.5, None)
    very_low = LO.attention(q, k, v, qpos, 0, d ** -0.5, np.full(nq, -1e4))
    assert np.array_equal(plain, very_low)
    sinks = np.array([0.5, -1.0, 2.0, 0.0])
    with_sink = LO.attention(q, k, v, qpos, 0, d ** -0.5, sinks).astype(np.float64)
    # the sink only rescales each row by sum(e) / (sum(e) + e^sink)
    for h in range(nq):
        s = (q[:, h].astype(np.float64) @ k[h // 2].astype(np.float64).T) * d ** -0.5
        s = np.where(np.arange(P)[None] <= qpos[:, None], s, -np.inf)
        m = np.maximum(s.max(1), sinks[h])
        e = np.exp(s - m[:, None]).sum(1)
        f = e / (e + np.exp(sinks[h] - m))
        assert np.allclose(with_sink[:, h], plain[:, h] * f[:, None], rtol=2e-2, atol=1e-3)


def test_window_mask_matches_a_loop():
    rng = np.random.default_rng(2)
    T, nq, nkv, d, P, W = 5, 2, 1, 8, 12, 4
    q, k, v = _bf(rng, T, nq, d), _bf(rng, nkv, P, d), _bf(rng, nkv, P, d)
    qpos = np.arange(P - T, P)
    got = LO.attention(q, k, v, qpos, W, 0.3, None)
    for t in range(T):
        for h in range(nq):
            js = [j for j in range(P) if qpos[t] - W < j <= qpos[t]]
            assert len(js) == W
            s = np.array([float(q[t, h].astype(np.float64) @ k[0, j].astype(np.float64)) * 0.3 for j in js])
            w = np.exp(s - s.max())
            ref = (w[:, None] * v[0, js].astype(np.float64)).sum(0) / w.sum()
            assert np.array_equal(got[t, h], bf16_round(ref.astype(np.float32)))


def _small_attn(window, sinks, seed=3, H=64):
    rng = np.random.default_rng(seed)
    nq, nkv, dqk, dv = 4, 2, 16, 8
    return LO.AttnWeights(wq=_bf(rng, nq * dqk, H, std=0.1), wk=_bf(rng, nkv * dqk, H, std=0.1),
                          wv=_bf(rng, nkv * dv, H, std=0.1), wo=_bf(rng, H, nq * dv, std=0.1),
                          sinks=rng.standard_normal(nq) if sinks else None, n_heads=nq, n_kv_heads=nkv,
                          head_dim=dqk, v_head_dim=dv, rotary_dim=8, rope_theta=10000.0, window=window,
                          v_scale=0.707)


@pytest.mark.parametrize("window,sinks", [(0, False), (5, True)])
def test_decode_equals_prefill_in_the_oracle(window, sinks):
    rng = np.random.default_rng(4)
    H, I = 64, 32
    a = _small_attn(window, sinks, H=H)
    wg, wu, wd = _bf(rng, I, H, std=0.1), _bf(rng, I, H, std=0.1), _bf(rng, H, I, std=0.1)
    mlp = lambda r: LO.dense_mlp(r, wg, wu, wd)  # noqa: E731
    x = _bf(rng, 12, H)
    c1 = LO.Cache(a)
    full = LO.decoder_layer(x, a, c1, mlp, None, None, 1e-5)
    c2 = LO.Cache(a)
    part = [LO.decoder_layer(x[:8], a, c2, mlp, None, None, 1e-5)]
    part += [LO.decoder_layer(x[t:t + 1], a, c2, mlp, None, None, 1e-5) for t in range(8, 12)]
    step = np.concatenate(part)
    assert np.abs(step - full).max() <= 2 ** -7 * np.abs(full).max()
    assert np.mean(step == full) > 0.99


def test_layer_entry_points_reject_bad_arguments_without_a_device():
    import mimo_moe
    L = mimo_moe.lib()
    EINVAL = 1
    p = 1 << 20  # never dereferenced: every call below fails its host-side checks first
    # unsupported head dims
    assert L.mimo_moe_layer_attention(p, p, p, None, 1, 64, 4, 96, 128, 0.1, 0, 0, 16, 1, p, None, 0, None, None) == EINVAL
    # heads not a multiple of the kv heads
    assert L.mimo_moe_layer_attention(p, p, p, None, 1, 63, 4, 192, 128, 0.1, 0, 0, 16, 1, p, None, 0, None, None) == EINVAL
    # full attention: pos0 + T beyond the cache
    assert L.mimo_moe_layer_attention(p, p, p, None, 4, 64, 4, 192, 128, 0.1, 0, 14, 16, 1, p, None, 0, None, None) == EINVAL
    # sliding window: window + T - 1 > cap
    assert L.mimo_moe_layer_attention(p, p, p, None, 8, 64, 8, 192, 128, 0.1, 128, 500, 130, 1, p, None, 0,
                                      None, None) == EINVAL
    # explicit splits without a workspace
    assert L.mimo_moe_layer_attention(p, p, p, None, 1, 64, 4, 192, 128, 0.1, 0, 100, 4096, 4, p, None, 0,
                                      None, None) == EINVAL
    # unaligned pointer
    assert L.mimo_moe_layer_attention(p + 2, p, p, None, 1, 64, 4, 192, 128, 0.1, 0, 0, 16, 1, p, None, 0,
                                      None, None) == EINVAL
    assert L.mimo_moe_layer_rope_store(p, 8, 64, 4, 192, 128, 65, 1e4, 0.0, 0, 16, p, p, p, None) == EINVAL  # odd rot
    assert L.mimo_moe_layer_rope_store(p, 32, 64, 4, 192, 128, 64, 1e4, 0.0, 0, 16, p, p, p, None) == EINVAL  # T>cap
    assert L.mimo_moe_layer_swiglu(p, 1, 12, p, None) == EINVAL
    assert L.mimo_moe_layer_add(p, p, 12, p, None) == EINVAL
    assert L.mimo_moe_layer_add_rmsnorm(p, p, None, 1, 4, 1e-5, p, p, None) == EINVAL
    assert L.mimo_moe_layer_attention_workspace_bytes(8, 64, 128, 1) == 0
    assert L.mimo_moe_layer_attention_workspace_bytes(8, 64, 128, 16) == 16 * 8 * 64 * (128 + 2) * 4


def test_decode_linear_host_checks_and_workspace_without_a_device():
    """mimo_moe_layer_linear's host side: argument checks before any launch, and the workspace its K split needs
    (one float32 partial row per token and output per segment; none when the weights split into one segment)."""
    import mimo_moe
    L = mimo_moe.lib()
    EINVAL = 1
    p = 1 << 20
    assert L.mimo_moe_layer_linear(p, p, 17, 4096, 4096, p, None, 0, None, None) == EINVAL   # T > 16
    assert L.mimo_moe_layer_linear(p, p, 8, 4100, 4096, p, None, 0, None, None) == EINVAL   # N % 8
    assert L.mimo_moe_layer_linear(p, p, 8, 4096, 4000, p, None, 0, None, None) == EINVAL   # K % 64
    assert L.mimo_moe_layer_linear(p, p, 8, 4096, 192, p, None, 0, None, None) == EINVAL    # K < 256
    assert L.mimo_moe_layer_linear(p + 2, p, 8, 4096, 4096, p, None, 0, None, None) == EINVAL
    assert L.mimo_moe_layer_linear_workspace_bytes(17, 4096, 4096) == 0
    for T, N, K in ((8, 13568, 4096), (1, 4096, 8192), (8, 32768, 4096), (8, 4096, 16384)):
        nb = L.mimo_moe_layer_linear_workspace_bytes(T, N, K)
        row = T * N * 4
        assert nb % row == 0 and nb // row in (0, 2, 4, 8, 16, 32)
        S = max(1, nb // row)
        assert K % (64 * S) == 0 and K // S >= 256


def test_attention_refuses_a_chunk_the_cache_cannot_hold_before_touching_it():
    """A chunk whose visible keys would not all fit the cache (full attention: past its end; sliding window:
    more than the ring holds) raises before the cache append, so the cache and its position are unchanged
    (host-side check, no device needed); the bound is the attention entry point's own."""
    import torch
    from mimo_moe.layer import Attention, KVCache, mimo_full_attention, mimo_sliding_attention
    for cfg, cap, offset, T in ((mimo_full_attention(), 256, 250, 8), (mimo_sliding_attention(), 256, 1000, 130)):
        H = 256
        wq = torch.zeros(cfg.n_heads * cfg.head_dim, H)
        wk = torch.zeros(cfg.n_kv_heads * cfg.head_dim, H)
        wv = torch.zeros(cfg.n_kv_heads * cfg.v_head_dim, H)
        wo = torch.zeros(H, cfg.n_heads * cfg.v_head_dim)
        attn = Attention(cfg, wq, wk, wv, wo, torch.zeros(cfg.n_heads) if cfg.sinks else None, device="cpu")
        cache = KVCache(cfg, cap, "cpu")
        cache.offset = offset
        with pytest.raises(ValueError, match="cache slots"):
            attn(torch.zeros(T, H, dtype=torch.bfloat16), cache)
        assert cache.offset == offset and not cache.k.any() and not cache.v.any()
    # the same bound as mimo_moe_layer_attention's (a ring shorter than window + T - 1 still takes a chunk
    # whose earliest visible key is position 0)
    import mimo_moe
    L = mimo_moe.lib()
    p = 1 << 20
    for window, pos0, T, cap, ok in ((128, 0, 8, 128, True), (128, 0, 129, 128, False), (128, 1000, 129, 256, True),
                                     (128, 1000, 130, 256, False), (0, 250, 6, 256, True), (0, 250, 7, 256, False)):
        first = max(0, pos0 - window + 1) if window > 0 else 0
        assert (pos0 + T - first <= cap) == ok
        if not ok:   # refused on the host, before any launch
            assert L.mimo_moe_layer_attention(p, p, p, None, T, 64, 8, 192, 128, 0.1, window, pos0, cap, 1, p, None,
                                              0, None, None) == 1
