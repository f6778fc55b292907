"""The rest of the MiMo decoder layer around the MoE block: attention with sinks (full or sliding window),
the dense MLP of the non-MoE layers, and the layer wrapper.

Mirrors engine/mimo_stream/mimo_v2.py (`Attention` :66-148, `MLP` :151-160, `DecoderLayer` :242-262) and the
engine's per-layer loop (engine/mimo_stream/model.py:294-300, caches from model.py:169-170):

    h   = x + self_attn(input_layernorm(x), mask, cache)
    out = h + mlp(post_attention_layernorm(h))          (mlp = the MoE block on MoE layers)

RoPE, the cache append, attention, the residual add fused with the next RMSNorm, the SwiGLU and the decode-size
projections (T <= 16 token rows) run in this library's CUDA kernels (include/mimo_moe_layer.h); prefill-sized
projections are plain bf16 GEMMs (cuBLAS through torch.matmul).  There is no CPU path.

The checkpoint's config.json is not available offline, so every dimension is a constructor argument;
`mimo_full_attention()` / `mimo_sliding_attention()` give the MiMo-like defaults the tests and the benchmark use
(hidden 4096, 64 query heads of 192 (q/k) and 128 (v) dims, 64 rotary dims, 4 kv heads on full-attention layers
and 8 on the 128-token sliding-window layers, sinks on the sliding-window layers)."""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Optional, Union

import torch

from ._lib import check, lib
from .ops import ExpertPools, _need_cuda, _ptr, _stream, moe_block, read_status, rmsnorm, workspace


@dataclass(frozen=True)
class AttentionConfig:
    """mimo_v2.py:68-83: the full-attention or sliding-window (swa_*) fields of ModelArgs."""
    n_heads: int = 64
    n_kv_heads: int = 4
    head_dim: int = 192
    v_head_dim: int = 128
    rotary_dim: int = 64            # int(partial_rotary_factor * head_dim)
    rope_theta: float = 5_000_000.0
    window: int = 0                 # sliding_window_size on SWA layers, 0 = full causal attention
    sinks: bool = False             # add_{full,swa}_attention_sink_bias
    v_scale: Optional[float] = None  # attention_value_scale

    @property
    def scale(self) -> float:
        return self.head_dim ** -0.5   # mimo_v2.py:92

    @property
    def qkv_width(self) -> int:
        return self.n_heads * self.head_dim + self.n_kv_heads * (self.head_dim + self.v_head_dim)


def mimo_full_attention(**kw) -> AttentionConfig:
    return replace(AttentionConfig(), **kw)


def mimo_sliding_attention(**kw) -> AttentionConfig:
    return replace(AttentionConfig(n_kv_heads=8, rope_theta=10_000.0, window=128, sinks=True), **kw)


def bf16_value(v: float) -> float:
    """The float a Python scalar becomes when MLX multiplies it into a bf16 array (cast to bf16)."""
    return float(torch.tensor(v, dtype=torch.float32).to(torch.bfloat16).to(torch.float32))


class KVCache:
    """Device KV cache of one attention layer: k [n_kv, cap, head_dim], v [n_kv, cap, v_head_dim] bf16,
    position p in slot p % cap.  Full attention: cap = the longest sequence (mlx_lm KVCache); sliding window:
    a ring of window + max_chunk - 1 slots (RotatingKVCache(max_size=window) keeps the last `window` keys and
    concatenates a multi-token chunk before trimming, which is what the extra max_chunk - 1 slots hold)."""

    def __init__(self, cfg: AttentionConfig, cap: int, device=None):
        dev = torch.device(device or "cuda")
        self.cfg = cfg
        self.cap = int(cap)
        self.k = torch.zeros(cfg.n_kv_heads, self.cap, cfg.head_dim, dtype=torch.bfloat16, device=dev)
        self.v = torch.zeros(cfg.n_kv_heads, self.cap, cfg.v_head_dim, dtype=torch.bfloat16, device=dev)
        self.offset = 0

    @classmethod
    def for_layer(cls, cfg: AttentionConfig, max_len: int, max_chunk: int = 4096, device=None) -> "KVCache":
        """Capacity rounded up to a multiple of 128 (the tcgen05 attention reads 128-key blocks that must not
        wrap around the ring)."""
        cap = max_len if cfg.window == 0 else min(max_len, cfg.window + max_chunk - 1)
        return cls(cfg, -(-cap // 128) * 128, device)


def rope_store(qkv: torch.Tensor, cfg: AttentionConfig, cache: KVCache, pos0: int,
               q_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """mimo_v2.py:130-139: RoPE on q and k at positions pos0.., v * attention_value_scale, k/v appended to the
    cache.  Returns q bf16 [T, n_heads, head_dim]."""
    _need_cuda(qkv, "qkv")
    qkv = qkv.to(torch.bfloat16).contiguous()
    T = qkv.shape[0]
    q = q_out if q_out is not None else torch.empty(T, cfg.n_heads, cfg.head_dim, dtype=torch.bfloat16,
                                                    device=qkv.device)
    vs = 0.0 if cfg.v_scale is None else bf16_value(cfg.v_scale)
    check(lib().mimo_moe_layer_rope_store(qkv.data_ptr(), T, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                                          cfg.v_head_dim, cfg.rotary_dim, float(cfg.rope_theta), vs, int(pos0),
                                          cache.cap, q.data_ptr(), cache.k.data_ptr(), cache.v.data_ptr(),
                                          _stream()), "rope_store")
    return q


def attention(q: torch.Tensor, cache: KVCache, cfg: AttentionConfig, pos0: int, sinks: Optional[torch.Tensor] = None,
              splits: int = 0, out: Optional[torch.Tensor] = None,
              status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """mlx fast.scaled_dot_product_attention(q, k, v, scale=head_dim^-0.5, mask, sinks) over the cache for the
    T queries at positions pos0..pos0+T-1 (causal; sliding window when cfg.window > 0).  Query tiles of 128
    rows run on the tcgen05 kernel (cache capacity a multiple of 128), decode-sized calls on the split-key
    mma.sync kernel.  Returns bf16 [T, n_heads, v_head_dim]."""
    _need_cuda(q, "q")
    q = q.to(torch.bfloat16).contiguous()
    T = q.shape[0]
    dev = q.device
    o = out if out is not None else torch.empty(T, cfg.n_heads, cfg.v_head_dim, dtype=torch.bfloat16, device=dev)
    L = lib()
    if splits <= 0:
        # the library's own choice never exceeds two CTAs per SM over the call's 64-row query tiles (prefill:
        # one split, no workspace)
        G = cfg.n_heads // cfg.n_kv_heads
        tiles = -(-T * G // 64)
        max_splits = min(64, -(-2 * 148 // (tiles * cfg.n_kv_heads)))
    else:
        max_splits = splits
    nb = L.mimo_moe_layer_attention_workspace_bytes(T, cfg.n_heads, cfg.v_head_dim, max_splits)
    ws = workspace(nb, dev) if nb else None
    if sinks is not None:
        sinks = sinks.to(device=dev, dtype=torch.float32).contiguous()
    check(L.mimo_moe_layer_attention(q.data_ptr(), cache.k.data_ptr(), cache.v.data_ptr(), _ptr(sinks), T,
                                     cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.v_head_dim, float(cfg.scale),
                                     cfg.window, int(pos0), cache.cap, int(splits), o.data_ptr(), _ptr(ws),
                                     ws.numel() if ws is not None else 0, _ptr(status), _stream()), "attention")
    return o


DECODE_ROWS = 16  # projections of at most this many token rows run on the library's decode kernel


def linear(x: torch.Tensor, weight: torch.Tensor, workspace_ok: bool = True) -> torch.Tensor:
    """nn.Linear without bias: x bf16 [T, K] . weight bf16 [N, K]^T -> bf16 [T, N].  Decode sizes (T <= 16) run
    on the library's tcgen05 stream kernel (mimo_moe_layer_linear, the weights read once); larger T are plain
    GEMMs on cuBLAS."""
    _need_cuda(x, "x")
    x = x.to(torch.bfloat16).contiguous()
    weight = weight.to(torch.bfloat16).contiguous()
    T, K = x.shape
    N = weight.shape[0]
    if weight.shape[1] != K:
        raise ValueError(f"linear: x has {K} features, weight expects {weight.shape[1]}")
    if T > DECODE_ROWS or N % 8 or K % 64 or K < 256:
        return torch.matmul(x, weight.t())
    y = torch.empty(T, N, dtype=torch.bfloat16, device=x.device)
    L = lib()
    nb = L.mimo_moe_layer_linear_workspace_bytes(T, N, K) if workspace_ok else 0
    ws = workspace(nb, x.device) if nb else None
    check(L.mimo_moe_layer_linear(x.data_ptr(), weight.data_ptr(), T, N, K, y.data_ptr(), _ptr(ws),
                                  ws.numel() if ws is not None else 0, None, _stream()), "linear")
    return y


def add_rmsnorm(x: torch.Tensor, delta: torch.Tensor, weight: Optional[torch.Tensor], eps: float):
    """h = bf16(x + delta), r = rmsnorm(h) * weight (one pass).  Returns (h, r)."""
    _need_cuda(x, "x")
    x = x.to(torch.bfloat16).contiguous()
    delta = delta.to(torch.bfloat16).contiguous()
    if delta.shape != x.shape:
        raise ValueError(f"add_rmsnorm: shapes {tuple(x.shape)} and {tuple(delta.shape)} differ")
    T, H = x.shape
    h = torch.empty_like(x)
    r = torch.empty_like(x)
    w = None if weight is None else weight.to(device=x.device, dtype=torch.bfloat16).contiguous()
    check(lib().mimo_moe_layer_add_rmsnorm(x.data_ptr(), delta.data_ptr(), _ptr(w), T, H, float(eps), h.data_ptr(),
                                           r.data_ptr(), _stream()), "add_rmsnorm")
    return h, r


def swiglu(gate_up: torch.Tensor) -> torch.Tensor:
    """mlx_lm swiglu(gate, up) = silu(gate) * up in bf16 steps; gate_up [T, 2I] = [gate | up]."""
    _need_cuda(gate_up, "gate_up")
    gate_up = gate_up.to(torch.bfloat16).contiguous()
    T, I2 = gate_up.shape
    out = torch.empty(T, I2 // 2, dtype=torch.bfloat16, device=gate_up.device)
    check(lib().mimo_moe_layer_swiglu(gate_up.data_ptr(), T, I2 // 2, out.data_ptr(), _stream()), "swiglu")
    return out


def add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """bf16(a + b), elementwise (the decoder layer's residual add)."""
    _need_cuda(a, "a")
    a = a.to(torch.bfloat16).contiguous()
    b = b.to(torch.bfloat16).contiguous()
    if a.shape != b.shape:
        raise ValueError(f"add: shapes {tuple(a.shape)} and {tuple(b.shape)} differ")
    out = torch.empty_like(a)
    check(lib().mimo_moe_layer_add(a.data_ptr(), b.data_ptr(), a.numel(), out.data_ptr(), _stream()), "add")
    return out


def _bf16(t: torch.Tensor, dev) -> torch.Tensor:
    return t.to(device=dev, dtype=torch.bfloat16).contiguous()


class Attention:
    """mimo_v2.py:66-148 (no attention bias).  Weights in nn.Linear layout [out, in]: wq [n_heads*head_dim, H],
    wk [n_kv*head_dim, H], wv [n_kv*v_head_dim, H], wo [H, n_heads*v_head_dim]; sinks float32 [n_heads]."""

    def __init__(self, cfg: AttentionConfig, wq, wk, wv, wo, sinks: Optional[torch.Tensor] = None, device=None):
        dev = torch.device(device or wq.device)
        if cfg.sinks and sinks is None:
            raise ValueError("this attention config has sinks: pass the sink logits")
        self.cfg = cfg
        self.w_qkv = torch.cat([_bf16(wq, dev), _bf16(wk, dev), _bf16(wv, dev)], 0).contiguous()
        self.w_o = _bf16(wo, dev)
        self.sinks = None if sinks is None else sinks.to(device=dev, dtype=torch.float32).contiguous()
        if self.w_qkv.shape[0] != cfg.qkv_width:
            raise ValueError("q/k/v weights do not match the attention config")

    def __call__(self, r: torch.Tensor, cache: KVCache) -> torch.Tensor:
        T = r.shape[0]
        cfg = self.cfg
        # the attention call's own check (every key visible to the chunk still in the ring), made before the
        # cache append so a refused chunk leaves the cache as it was
        first = max(0, cache.offset - cfg.window + 1) if cfg.window > 0 else 0
        need = cache.offset + T - first
        if need > cache.cap:
            raise ValueError(f"attention: {T} tokens at position {cache.offset} need {need} cache slots; the cache "
                             f"has {cache.cap}")
        qkv = linear(r, self.w_qkv)
        q = rope_store(qkv, self.cfg, cache, cache.offset)
        o = attention(q, cache, self.cfg, cache.offset, self.sinks)
        cache.offset += T
        return linear(o.view(T, -1), self.w_o)


class DenseMLP:
    """mimo_v2.py:151-160: down(swiglu(gate(x), up(x))); weights [I, H], [I, H], [H, I]."""

    def __init__(self, w_gate, w_up, w_down, device=None):
        dev = torch.device(device or w_gate.device)
        self.w_gate_up = torch.cat([_bf16(w_gate, dev), _bf16(w_up, dev)], 0).contiguous()
        self.w_down = _bf16(w_down, dev)

    def __call__(self, r: torch.Tensor) -> torch.Tensor:
        return linear(swiglu(linear(r, self.w_gate_up)), self.w_down)


class MoEMLP:
    """An MoE layer's MLP: the router + resident experts of this library's MoE block (model.py:302-336).
    The block's device status word lives with the layer (zeroed once; the first error stays until
    check_status() reads and clears it), so a step launches no per-call fill."""

    def __init__(self, router_weight: torch.Tensor, bias: Optional[torch.Tensor], pools: ExpertPools):
        self.router_weight = router_weight.to(torch.bfloat16).contiguous()
        self.bias = None if bias is None else bias.to(torch.float32).contiguous()
        self.pools = pools
        self.status = torch.zeros(1, dtype=torch.int32, device=self.router_weight.device)

    def __call__(self, r: torch.Tensor) -> torch.Tensor:
        return moe_block(r, self.router_weight, self.bias, self.pools, status=self.status)

    def check_status(self) -> None:
        """Synchronise on the status word; raise like the reference for a bad route, then clear it."""
        try:
            read_status(self.status, "MoE layer")
        finally:
            self.status.zero_()


class DecoderLayer:
    """mimo_v2.py:242-262: h = x + attn(input_layernorm(x)); out = h + mlp(post_attention_layernorm(h)).
    __call__(x bf16 [T, H], cache) -> bf16 [T, H]; the cache's offset advances by T."""

    def __init__(self, attn: Attention, mlp: Union[DenseMLP, MoEMLP], input_norm: Optional[torch.Tensor],
                 post_norm: Optional[torch.Tensor], eps: float = 1e-5):
        self.attn = attn
        self.mlp = mlp
        dev = attn.w_o.device
        self.input_norm = None if input_norm is None else _bf16(input_norm, dev)
        self.post_norm = None if post_norm is None else _bf16(post_norm, dev)
        self.eps = float(eps)
        self.trace = None   # optional callable(dict of the layer's intermediate tensors), for tests

    def new_cache(self, max_len: int, max_chunk: int = 4096) -> KVCache:
        return KVCache.for_layer(self.attn.cfg, max_len, max_chunk, self.attn.w_o.device)

    def parts(self, x: torch.Tensor, cache: KVCache, r: Optional[torch.Tensor] = None):
        """The layer up to its last residual add: returns (h, y) with out = bf16(h + y).  r, when given, is
        input_layernorm(x) already computed (a stack folds it into the previous layer's last add)."""
        if r is None:
            r = rmsnorm(x, self.input_norm, self.eps)
        a = self.attn(r, cache)
        h, r2 = add_rmsnorm(x, a, self.post_norm, self.eps)
        y = self.mlp(r2)
        if self.trace is not None:
            self.trace({"x": x, "r": r, "a": a, "h": h, "r2": r2, "y": y})
        return h, y

    def __call__(self, x: torch.Tensor, cache: KVCache) -> torch.Tensor:
        _need_cuda(x, "x")
        x = x.to(torch.bfloat16).contiguous()
        h, y = self.parts(x, cache)
        return add(h, y)


class DecoderStack:
    """Decoder layers run in order over one residual stream (the engine's layer loop, model.py:294-336, without
    the embedding, final norm and lm_head): each layer's KV cache lives here, every layer of a call works at
    the same position, each layer's last residual add runs together with the next layer's input norm (one
    add + RMSNorm pass, bit-identical to the two), and the output is a fixed buffer per shape, so a decode
    step replays as one CUDA graph (the graph keeps the position it was captured at; `at(pos)` sets it for
    eager calls and captures)."""

    def __init__(self, layers, max_len: int, max_chunk: int = 4096):
        if not layers:
            raise ValueError("empty stack")
        self.layers = list(layers)
        self.caches = [l.new_cache(max_len, max_chunk) for l in self.layers]
        self._out = {}

    def at(self, pos: int) -> "DecoderStack":
        for c in self.caches:
            c.offset = int(pos)
        return self

    @property
    def offset(self) -> int:
        return self.caches[0].offset

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        _need_cuda(x, "x")
        h = x.to(torch.bfloat16).contiguous()
        r = None
        n = len(self.layers)
        for i, (layer, cache) in enumerate(zip(self.layers, self.caches)):
            hh, y = layer.parts(h, cache, r)
            if i + 1 < n:   # this layer's residual add and the next layer's input norm in one pass
                nxt = self.layers[i + 1]
                h, r = add_rmsnorm(hh, y, nxt.input_norm, nxt.eps)
            else:
                h = add(hh, y)
        key = (tuple(h.shape), h.device)
        if key not in self._out:
            self._out[key] = torch.empty_like(h)
        out = self._out[key]
        out.copy_(h)
        return out


def synthetic_attention(cfg: AttentionConfig, hidden: int = 4096, seed: int = 4, std: float = 0.02,
                        device=None, on_device: bool = False) -> Attention:
    """Seeded random-init attention weights of this shape (no checkpoint offline): N(0, std) bf16, sinks
    N(0, 1) float32 when the config has them.  on_device draws them with a CUDA generator (fast, for
    benchmark-sized stacks) instead of the CPU generator the tests use."""
    dev = torch.device(device or "cuda")
    gdev = dev if on_device else torch.device("cpu")
    g = torch.Generator(gdev).manual_seed(seed)
    def w(o, i):
        return (torch.randn(o, i, generator=g, device=gdev) * std).to(torch.bfloat16)
    wq = w(cfg.n_heads * cfg.head_dim, hidden)
    wk = w(cfg.n_kv_heads * cfg.head_dim, hidden)
    wv = w(cfg.n_kv_heads * cfg.v_head_dim, hidden)
    wo = w(hidden, cfg.n_heads * cfg.v_head_dim)
    sinks = torch.randn(cfg.n_heads, generator=g, device=gdev) if cfg.sinks else None
    return Attention(cfg, wq, wk, wv, wo, sinks, device=dev)


def synthetic_dense_mlp(hidden: int = 4096, inter: int = 16384, seed: int = 5, std: float = 0.02,
                        device=None, on_device: bool = False) -> DenseMLP:
    dev = torch.device(device or "cuda")
    gdev = dev if on_device else torch.device("cpu")
    g = torch.Generator(gdev).manual_seed(seed)
    def w(o, i):
        return (torch.randn(o, i, generator=g, device=gdev) * std).to(torch.bfloat16)
    return DenseMLP(w(inter, hidden), w(inter, hidden), w(hidden, inter), device=dev)


__all__ = ["AttentionConfig", "Attention", "DecoderLayer", "DecoderStack", "DenseMLP", "KVCache", "MoEMLP", "add",
           "add_rmsnorm", "attention", "linear", "bf16_value", "mimo_full_attention", "mimo_sliding_attention", "rope_store", "swiglu",
           "synthetic_attention", "synthetic_dense_mlp"]
