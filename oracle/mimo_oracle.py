"""CPU oracle for the MiMo MoE block (router -> dispatch -> MXFP4 experts -> combine).

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library imports this module: only `tests/`,
`__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of `bench.py` use it, and
there only as the checker (or as the timed CPU restatement of the reference path).

It restates, in numpy, the reference's per-layer expert path of `engine/mimo_stream` (paths relative to
the reference project root):

  * router ............ engine/mimo_stream/model.py:58-65   (FP32 logits, sigmoid, noaux bias, top-8,
                                                               weights = unbiased scores / (sum + 1e-20))
  * MXFP4 decode ...... engine/mimo_stream/kernels.py:19-30 (e2m1 nibble, e8m0 scale; s=0 -> 2^-127,
                                                               s=255 -> NaN; low nibble first)
  * sigmoid LUT ....... engine/mimo_stream/kernels.py:138-146 (bf16 sigmoid of every bf16 bit pattern)
  * route grouping .... engine/mimo_stream/kernels.py:149-173 (group_routes)
  * kernel A .......... engine/mimo_stream/kernels.py:33-85  (gate/up dots, bf16(g), bf16(u),
                                                               h = bf16(bf16(g*sig[g]) * u))
  * kernel B .......... engine/mimo_stream/kernels.py:88-123 (part = fp32(down . h) * w)
  * combine ........... engine/mimo_stream/kernels.py:194-199 (gather by gather_idx, fixed-order sum)
  * M=1 path .......... engine/mimo_stream/model.py:173-182  (gather_qmm x3: bf16 outputs, fp32 weighted sum)
  * prefill path ...... engine/mimo_stream/model.py:221-271  (stable argsort by slot, pair products,
                                                               inverse permutation, fp32 weighted sum)
  * fp32 reference .... engine/tests/test_kernels.py:32-46, rel_err at :54-56

Rounding points that the reference leaves to MLX internals (the order of the simd_sum, MLX's matmul and
reduction order, MLX's bf16 sigmoid) are "parity unpinned" at the ulp level: this oracle evaluates each
dot product in float64 and rounds once to float32 at the point where the reference holds a float32, and
defines the sigmoid table as the correctly rounded bf16 of the exact sigmoid.  The reference's own tests
pin only a tolerance at this boundary (test_kernels.py:79,89: rel_err < 2e-2 against FP32 dequant).

Top-k order.  MLX `argpartition` returns the top-8 in an unspecified order (model.py:62) and the combine
sums in that order.  This build fixes a total order: descending selection score, ties broken by
ascending expert id.  Router weights are normalised by a float32 sum taken in that order.
"""
from __future__ import annotations

import numpy as np

H, I, E, TOPK, R = 4096, 2048, 256, 8, 8
GROUP = 32
SHAPES = {"gate": (I, H), "up": (I, H), "down": (H, I)}          # (out, in); model.py:28
EXPERT_BYTES = sum(o * i // 2 + o * i // 32 for o, i in SHAPES.values())   # 13,369,344; model.py:29

# e2m1 code -> value (sign bit 3, magnitude table indexed by code & 7); kernels.py:21-23
E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                 -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], np.float32)


# ----------------------------------------------------------------------------------------- bf16 helpers
def f32_to_bf16_bits(a) -> np.ndarray:
    """Round float32 to bfloat16 (round to nearest even), returned as uint16 bit patterns."""
    a = np.ascontiguousarray(np.asarray(a, np.float32))
    b = a.view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint32)
    nan = np.isnan(a)
    r[nan] = 0x7FC0
    return r.astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(a) -> np.ndarray:
    """float32 -> bf16 -> float32 (round to nearest even)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


# ------------------------------------------------------------------------------------------ MXFP4 decode
def e8m0_to_f32(s) -> np.ndarray:
    """e8m0 byte -> 2^(s-127); s=0 -> 2^-127, s=255 -> NaN (kernels.py:24-29)."""
    s = np.asarray(s, np.uint8).astype(np.uint32)
    out = (s << 23).view(np.float32).copy()
    out[s == 0] = np.float32(2.0 ** -127)
    out[s == 255] = np.nan
    return out


def unpack_e2m1(words: np.ndarray) -> np.ndarray:
    """uint32 [..., n/8] -> float32 [..., n]; element k is nibble k%8 of word k/8 (low nibble first)."""
    w = np.asarray(words, np.uint32)
    nib = (w[..., None] >> (4 * np.arange(8, dtype=np.uint32))) & 0xF
    return E2M1[nib.reshape(*w.shape[:-1], w.shape[-1] * 8)]


def dequant(words: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """MXFP4 [.., out, in/8] u32 + [.., out, in/32] u8 -> float32 [.., out, in]."""
    v = unpack_e2m1(words)
    sc = e8m0_to_f32(scales)
    shp = v.shape
    v = v.reshape(*shp[:-1], shp[-1] // GROUP, GROUP) * sc[..., None]
    return v.reshape(shp)


_BYTE_LUT = np.stack([E2M1[np.arange(256) & 15], E2M1[np.arange(256) >> 4]], 1).astype(np.float64)


def dequant64(words: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Same values as dequant(), produced in float64 through a byte -> (even, odd) element table."""
    w = np.ascontiguousarray(np.asarray(words, np.uint32))
    v = _BYTE_LUT[w.view(np.uint8)]                       # [.., in/2, 2]
    shp = w.shape[:-1] + (w.shape[-1] * 8,)
    v = v.reshape(*shp[:-1], shp[-1] // GROUP, GROUP)
    v *= e8m0_to_f32(scales).astype(np.float64)[..., None]
    return v.reshape(shp)


_SIGTAB = None


def sigmoid_table() -> np.ndarray:
    """bf16 sigmoid for every bf16 bit pattern (kernels.py:138-146), as float32 values.

    Defined here as the correctly rounded bf16 of the exact sigmoid (computed in float64)."""
    global _SIGTAB
    if _SIGTAB is None:
        with np.errstate(over="ignore", invalid="ignore"):
            v = bf16_bits_to_f32(np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)).astype(np.float64)
            s = 1.0 / (1.0 + np.exp(-v))
        _SIGTAB = bf16_round(s.astype(np.float32))
    return _SIGTAB


def sigmoid_table_bits() -> np.ndarray:
    return f32_to_bf16_bits(sigmoid_table())


def swiglu_bf16(g32: np.ndarray, u32: np.ndarray) -> np.ndarray:
    """Kernel A's epilogue (kernels.py:79-82): gt=bf16(g), ut=bf16(u), h = bf16(bf16(gt*sig[gt])*ut)."""
    gt = f32_to_bf16_bits(g32)
    ut = bf16_bits_to_f32(f32_to_bf16_bits(u32))
    sig = sigmoid_table()[gt]
    gs = bf16_round(bf16_bits_to_f32(gt) * sig)
    return bf16_round(gs * ut)


# ---------------------------------------------------------------------------------------------- router
def sigmoid_f32(logits: np.ndarray) -> np.ndarray:
    """Sigmoid evaluated in float64 and rounded once to float32."""
    l64 = np.asarray(logits, np.float32).astype(np.float64)
    with np.errstate(over="ignore"):
        return (1.0 / (1.0 + np.exp(-l64))).astype(np.float32)


def router_logits(x: np.ndarray, W: np.ndarray) -> np.ndarray:
    """FP32 logits = fp32(x) @ fp32(W).T (model.py:59), evaluated in float64 and rounded to float32."""
    return (np.asarray(x, np.float64) @ np.asarray(W, np.float64).T).astype(np.float32)


def topk_from_logits(logits: np.ndarray, bias: np.ndarray, k: int = TOPK):
    """model.py:60-64 with a total order: sel desc, then expert id asc.  NaN selection scores sort last.

    Returns (inds int32 [T,k], w float32 [T,k]) with w = s[inds] / (sum_k s[inds] + 1e-20), the sum
    taken in float32 in output order."""
    logits = np.asarray(logits, np.float32)
    T, n = logits.shape
    s = sigmoid_f32(logits)
    sel = (s + np.asarray(bias, np.float32)[None, :]).astype(np.float32)
    key = np.where(np.isnan(sel), -np.inf, sel)
    ids = np.broadcast_to(np.arange(n), (T, n))
    order = np.lexsort((ids, -key), axis=-1)[:, :k]
    inds = order.astype(np.int32)
    ws = np.take_along_axis(s, order, axis=-1).astype(np.float32)
    tot = np.zeros(T, np.float32)
    for j in range(k):
        tot = (tot + ws[:, j]).astype(np.float32)
    tot = (tot + np.float32(1e-20)).astype(np.float32)
    return inds, (ws / tot[:, None]).astype(np.float32)


def router(x: np.ndarray, W: np.ndarray, bias: np.ndarray, k: int = TOPK):
    """Router.__call__ (model.py:58-65).  x float32 values of bf16 [T,H]; W float32 values of bf16."""
    logits = router_logits(x, W)
    inds, w = topk_from_logits(logits, bias, k)
    return logits, inds, w


# -------------------------------------------------------------------------------------------- dispatch
def group_routes(inds: np.ndarray, scores: np.ndarray, R: int = R):
    """Restatement of kernels.py:149-173.  Distinct experts ascending; per expert, routes in flat
    (row, k) order up to R; gather_idx[t] = u*R + c.  Raises ValueError when more than R rows hit one
    expert (kernels.py:167-168)."""
    inds = np.asarray(inds)
    M, k = inds.shape
    flat = inds.reshape(-1)
    uids, inv = np.unique(flat, return_inverse=True)
    U = len(uids)
    urows = np.zeros((U, R), np.int32)
    uw = np.zeros((U, R), np.float32)
    ucnt = np.zeros(U, np.int32)
    rows = np.repeat(np.arange(M), k)
    sc = np.asarray(scores, np.float32).reshape(-1)
    gidx = np.zeros(flat.size, np.uint32)
    for t in range(flat.size):
        u = inv[t]
        c = ucnt[u]
        if c >= R:
            raise ValueError("more rows than R routed to one expert")
        urows[u, c] = rows[t]
        uw[u, c] = sc[t]
        gidx[t] = u * R + c
        ucnt[u] = c + 1
    return uids, urows, ucnt, uw, gidx


def dispatch(inds: np.ndarray, n_experts: int = E):
    """Prefill permutation (model.py:235-244, 266-268): pairs (token, k) in flat order, stable-argsorted
    by expert; inv[order] = arange.  Returns (offsets int32 [E+1], order int32 [P], inv int32 [P])."""
    flat = np.asarray(inds).reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable").astype(np.int32)
    inv = np.empty_like(order)
    inv[order] = np.arange(order.size, dtype=np.int32)
    counts = np.bincount(flat, minlength=n_experts)
    offsets = np.zeros(n_experts + 1, np.int32)
    offsets[1:] = np.cumsum(counts)
    return offsets, order, inv


# -------------------------------------------------------------------------------------------- experts
class Pool:
    """Expert pool {gate,up,down}_{w,s} in the reference layout (model.py:32-45), with a bounded LRU
    cache of dequantised experts (float64 holds every MXFP4 value exactly).  `arrays` may be numpy
    arrays or any object whose arrays[name][e] returns expert e's slice."""

    def __init__(self, arrays, cache: int = 6):
        self.a = arrays
        self._cache = {}
        self._limit = cache

    def deq(self, e: int):
        e = int(e)
        if e in self._cache:
            self._cache[e] = self._cache.pop(e)
            return self._cache[e]
        d = {n: dequant64(np.asarray(self.a[f"{n}_w"][e]), np.asarray(self.a[f"{n}_s"][e]))
             for n in ("gate", "up", "down")}
        self._cache[e] = d
        while len(self._cache) > self._limit:
            self._cache.pop(next(iter(self._cache)))
        return d

    def drop(self):
        self._cache.clear()


def _dots32(Wf: np.ndarray, X: np.ndarray) -> np.ndarray:
    """Rows of X [n, K] dotted with every row of Wf [N, K] in float64, rounded once to float32 ->
    [n, N] (the value a float32-accumulating kernel approximates)."""
    return (np.asarray(X, np.float64) @ np.asarray(Wf, np.float64).T).astype(np.float32)


def _expert_h(d, X: np.ndarray) -> np.ndarray:
    """Kernel A for the rows X [n, H] of one expert: h [n, I] (bf16 values)."""
    return swiglu_bf16(_dots32(d["gate"], X), _dots32(d["up"], X))


def moe_experts(x: np.ndarray, pool: Pool, uslot, urows, ucnt, uw, R: int = R, gather_idx=None):
    """kernels.py:176-199 (kernels A and B + combine).  x float32 values of bf16 [M,H].  Returns float32
    values of the bf16 output [M,H]."""
    x = np.asarray(x, np.float32)
    M = x.shape[0]
    U = len(uslot)
    Hd = x.shape[1]
    part = np.zeros((U, R, Hd), np.float32)
    for u in range(U):
        c = int(ucnt[u])
        if c == 0:
            continue
        d = pool.deq(uslot[u])
        rows = np.asarray(urows[u][:c], np.int64)
        h = _expert_h(d, x[rows])
        dn = _dots32(d["down"], h)                                   # [c, H]
        part[u, :c] = (dn * np.asarray(uw[u][:c], np.float32)[:, None]).astype(np.float32)
    if gather_idx is None:      # kernels.py:196-197 (scatter-add; summed here in (u, r) order)
        y = np.zeros((M, Hd), np.float32)
        for u in range(U):
            for r in range(int(ucnt[u])):
                y[int(urows[u][r])] = (y[int(urows[u][r])] + part[u, r]).astype(np.float32)
        return bf16_round(y)
    Y = part.reshape(-1, Hd)[np.asarray(gather_idx, np.int64)].reshape(M, -1, Hd)
    acc = np.zeros((M, Hd), np.float32)
    for j in range(Y.shape[1]):
        acc = (acc + Y[:, j]).astype(np.float32)
    return bf16_round(acc)


def pair_outputs(pool: Pool, e: int, X: np.ndarray) -> np.ndarray:
    """(token, expert) products of the gather_qmm path (model.py:179-181, 226-228) for the token rows
    X [n, H] of expert e: a, b and the down output are bf16; silu(a)*b in bf16 (the sigmoid table
    stands in for MLX's bf16 sigmoid)."""
    d = pool.deq(e)
    return bf16_round(_dots32(d["down"], _expert_h(d, X)))


def moe_pairs(x: np.ndarray, pool: Pool, inds, w):
    """M=1 path (model.py:173-182) and prefill path (model.py:221-271) with all experts resident:
    y[t] = bf16(sum_k fp32(pair(t, k)) * w[t, k]), summed over k in route order."""
    x = np.asarray(x, np.float32)
    inds = np.asarray(inds)
    T, k = inds.shape
    offsets, order, inv = dispatch(inds, max(E, int(inds.max()) + 1))
    tok = np.repeat(np.arange(T), k)
    flat = inds.reshape(-1)
    outs = np.zeros((T * k, x.shape[1]), np.float32)
    for e in np.unique(flat):          # slot-sorted pair order, as _pair_outputs consumes it
        ps = order[offsets[e]:offsets[e + 1]]
        outs[ps] = pair_outputs(pool, int(e), x[tok[ps]])
    Y = outs.reshape(T, k, -1)
    acc = np.zeros((T, Y.shape[-1]), np.float32)
    wf = np.asarray(w, np.float32)
    for j in range(k):
        acc = (acc + (Y[:, j] * wf[:, j:j + 1]).astype(np.float32)).astype(np.float32)
    return bf16_round(acc)


def moe_layer(x, pool: Pool, inds, w, R: int = R):
    """The reference's dispatch rule (model.py:184-219, 324-336): T==1 -> gather_qmm path,
    2<=T<=8 -> grouped kernels, T>8 -> prefill path."""
    T = np.asarray(x).shape[0]
    if T == 1 or T > 8:
        return moe_pairs(x, pool, inds, w)
    uids, urows, ucnt, uw, gidx = group_routes(inds, w, R)
    return moe_experts(x, pool, uids, urows, ucnt, uw, R, gather_idx=gidx)


def reference_fp32(x, pool: Pool, inds, scores):
    """test_kernels.py:32-46: FP32 dequant, g=Wg x, u=Wu x, h=g*sigmoid(g)*u, acc += s*(Wd h)
    (evaluated in float64, grouped by expert; the per-row sum runs in route order)."""
    x = np.asarray(x, np.float64)
    inds = np.asarray(inds)
    T, k = inds.shape
    contrib = np.zeros((T, k, x.shape[1]), np.float64)
    for e in np.unique(inds):
        t_idx, j_idx = np.nonzero(inds == e)
        d = pool.deq(int(e))
        X = x[t_idx]
        g = X @ d["gate"].T
        u = X @ d["up"].T
        hh = g / (1.0 + np.exp(-g)) * u
        contrib[t_idx, j_idx] = (hh @ d["down"].T) * \
            np.asarray(scores, np.float64)[t_idx, j_idx][:, None]
    return contrib.sum(axis=1).astype(np.float32)


def rel_err(a, b) -> float:
    """test_kernels.py:54-56: max|a-b| / (max|b| + 1e-9)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-9))


def moe_block(x, W, bias, pool: Pool, R: int = R):
    """Router + reference dispatch rule, end to end."""
    logits, inds, w = router(x, W, bias)
    return logits, inds, w, moe_layer(x, pool, inds, w, R)


def rmsnorm(x, weight=None, eps: float = 1e-6) -> np.ndarray:
    """model.py:75 (`nn.RMSNorm`, MLX fast.rms_norm): y = bf16(x * rsqrt(mean(x^2) + eps)) [* weight].
    Sum of squares exact in float64, rounded to float32; mean, +eps and rsqrt each rounded to float32
    (MLX's own float32 reduction order is parity unpinned at the ulp level)."""
    x32 = np.asarray(x, np.float32)
    ss = np.sum(x32.astype(np.float64) ** 2, axis=-1).astype(np.float32)
    ms = (ss / np.float32(x32.shape[-1])).astype(np.float32)
    v = (ms + np.float32(eps)).astype(np.float32)
    inv = (1.0 / np.sqrt(v.astype(np.float64))).astype(np.float32)
    y = bf16_round(x32 * inv[..., None])
    if weight is not None:
        y = bf16_round(np.asarray(weight, np.float32) * y)
    return y


def moe_stack(x, layers, eps: float = 1e-6, R: int = R):
    """BASELINE.json config 3's decode stack: x_{l+1} = rmsnorm(moe_block_l(x_l)) between layers, unit weight;
    returns the last layer's MoE output and every layer's routes.  layers: [(W, bias, Pool), ...]."""
    routes = []
    y = None
    for li, (W, bias, pool) in enumerate(layers):
        if li:
            x = rmsnorm(y, None, eps)
        _, inds, w, y = moe_block(x, W, bias, pool, R)
        routes.append(inds)
    return y, routes
