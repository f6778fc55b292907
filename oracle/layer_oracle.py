"""CPU oracle for the rest of the MiMo decoder layer (attention with sinks, dense MLP, residual adds, norms).

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library imports this module: only `tests/` and the CPU legs
of `bench.py` use it, as the checker.

It restates, in numpy (float64 arithmetic, rounded to float32 / bf16 where the reference holds those types):

  * decoder layer ..... engine/mimo_stream/mimo_v2.py:242-262 (h = x + attn(norm(x)); out = h + mlp(norm(h)));
                         the engine's loop engine/mimo_stream/model.py:294-300 (same composition)
  * attention ......... mimo_v2.py:110-148 (q/k/v projections, value scale, RoPE with the cache offset,
                         scaled_dot_product_attention with `sinks`, o_proj)
  * caches / masks .... model.py:169-170 (KVCache for full layers, RotatingKVCache(max_size=window) for
                         sliding-window layers), model.py:297 (create_attention_mask with window_size)
  * dense MLP ......... mimo_v2.py:151-160 (down(swiglu(gate(x), up(x))))

The operators behind these lines live in MLX 0.32.2 and mlx-lm 0.31.3 (pinned in the reference's
requirements.txt:2-3, not vendored, not installable offline).  Their published semantics, restated here:
  * nn.Linear on bf16: float32 accumulation, bf16 result (the accumulation order is MLX's: parity unpinned at
    the ulp level; here every dot product is exact in float64 and rounded once to float32, then to bf16);
  * nn.RoPE(dims, traditional=False, base): the pair (x[i], x[i + dims/2]), i < dims/2, rotated by
    pos * base^(-2i/dims); the remaining dims unchanged; bf16 in, bf16 out (MLX computes in float32);
  * fast.scaled_dot_product_attention(q, k, v, scale, mask, sinks): softmax over the scaled scores of the
    visible keys with one extra logit sinks[h] (no value row), GQA head h -> kv head h // (n_heads / n_kv);
  * create_attention_mask(..., window_size=w): key j visible to query i when j <= i and j > i - w;
  * swiglu(g, u) = silu(g) * u with silu(g) = g * sigmoid(g), each op rounded to bf16.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

from .mimo_oracle import bf16_round, rmsnorm, swiglu_bf16


def bf16(a) -> np.ndarray:
    return bf16_round(np.asarray(a, np.float64).astype(np.float32))


def linear(x: np.ndarray, W: np.ndarray) -> np.ndarray:
    """nn.Linear without bias: x [T, in], W [out, in] (bf16 values) -> bf16 [T, out]."""
    return bf16(np.asarray(x, np.float64) @ np.asarray(W, np.float64).T)


def rope(x: np.ndarray, positions: np.ndarray, rotary_dim: int, base: float) -> np.ndarray:
    """nn.RoPE(rotary_dim, traditional=False, base) on x [T, heads, d] at the given absolute positions."""
    x64 = np.asarray(x, np.float64)
    out = x64.copy()
    half = rotary_dim // 2
    i = np.arange(half, dtype=np.float64)
    inv_freq = np.exp(-(2.0 * i) / rotary_dim * np.log(float(np.float32(base))))
    ang = np.asarray(positions, np.float64)[:, None] * inv_freq[None, :]          # [T, half]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    x1, x2 = x64[..., :half], x64[..., half:rotary_dim]
    out[..., :half] = x1 * c - x2 * s
    out[..., half:rotary_dim] = x1 * s + x2 * c
    return bf16(out)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, qpos: np.ndarray, window: int, scale: float,
              sinks: Optional[np.ndarray] = None) -> np.ndarray:
    """q [T, nq, dqk]; k [nkv, P, dqk], v [nkv, P, dv] hold positions 0..P-1; qpos [T] absolute positions.
    Returns bf16 [T, nq, dv]."""
    T, nq, _ = q.shape
    nkv, P, _ = k.shape
    dv = v.shape[2]
    G = nq // nkv
    out = np.zeros((T, nq, dv), np.float64)
    kpos = np.arange(P)
    for hk in range(nkv):
        K = np.asarray(k[hk], np.float64)
        V = np.asarray(v[hk], np.float64)
        for g in range(G):
            h = hk * G + g
            s = (np.asarray(q[:, h], np.float64) @ K.T) * scale                       # [T, P]
            vis = kpos[None, :] <= qpos[:, None]
            if window > 0:
                vis &= kpos[None, :] > qpos[:, None] - window
            s = np.where(vis, s, -np.inf)
            m = s.max(axis=1)
            if sinks is not None:
                m = np.maximum(m, float(sinks[h]))
            e = np.exp(s - m[:, None])
            den = e.sum(axis=1)
            if sinks is not None:
                den = den + np.exp(float(sinks[h]) - m)
            out[:, h] = (e @ V) / den[:, None]
    return bf16(out)


@dataclass
class AttnWeights:
    wq: np.ndarray   # [nq*dqk, H]  (bf16 values as float32)
    wk: np.ndarray
    wv: np.ndarray
    wo: np.ndarray   # [H, nq*dv]
    sinks: Optional[np.ndarray]
    n_heads: int
    n_kv_heads: int
    head_dim: int
    v_head_dim: int
    rotary_dim: int
    rope_theta: float
    window: int
    v_scale: Optional[float]


class Cache:
    """Every position's k and v (the oracle keeps them all; the window is applied by the mask)."""

    def __init__(self, a: AttnWeights):
        self.k = np.zeros((a.n_kv_heads, 0, a.head_dim), np.float32)
        self.v = np.zeros((a.n_kv_heads, 0, a.v_head_dim), np.float32)

    @property
    def offset(self) -> int:
        return self.k.shape[1]


def attention_block(r: np.ndarray, a: AttnWeights, cache: Cache) -> np.ndarray:
    """mimo_v2.py:110-148 for T tokens appended to the cache; returns o_proj output bf16 [T, H]."""
    T = r.shape[0]
    pos0 = cache.offset
    q = linear(r, a.wq).reshape(T, a.n_heads, a.head_dim)
    kk = linear(r, a.wk).reshape(T, a.n_kv_heads, a.head_dim)
    vv = linear(r, a.wv).reshape(T, a.n_kv_heads, a.v_head_dim)
    if a.v_scale is not None:
        vv = bf16(vv * float(bf16(np.array([a.v_scale], np.float32))[0]))
    pos = np.arange(pos0, pos0 + T)
    q = rope(q, pos, a.rotary_dim, a.rope_theta)
    kk = rope(kk, pos, a.rotary_dim, a.rope_theta)
    cache.k = np.concatenate([cache.k, kk.transpose(1, 0, 2)], axis=1)
    cache.v = np.concatenate([cache.v, vv.transpose(1, 0, 2)], axis=1)
    o = attention(q, cache.k, cache.v, pos, a.window, a.head_dim ** -0.5, a.sinks)
    return linear(o.reshape(T, -1), a.wo)


def dense_mlp(r: np.ndarray, w_gate: np.ndarray, w_up: np.ndarray, w_down: np.ndarray) -> np.ndarray:
    g = linear(r, w_gate)
    u = linear(r, w_up)
    return linear(swiglu_bf16(g, u), w_down)


def add(a, b) -> np.ndarray:
    """bf16 + bf16 -> bf16 (float32 add, rounded)."""
    return bf16_round(np.asarray(a, np.float32) + np.asarray(b, np.float32))


def decoder_layer(x: np.ndarray, a: AttnWeights, cache: Cache, mlp, in_norm, post_norm, eps: float):
    """mimo_v2.py:258-262.  mlp: a callable r2 -> y (dense MLP or the MoE block oracle)."""
    r = rmsnorm(x, in_norm, eps)
    h = add(x, attention_block(r, a, cache))
    r2 = rmsnorm(h, post_norm, eps)
    return add(h, mlp(r2))
