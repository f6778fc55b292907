"""Batched CPU restatement of the pair path, for parity checks at the BASELINE.json sizes.

TEST INFRASTRUCTURE ONLY (imported by `tests/` and the CPU legs of `bench.py`, never by the library).

The arithmetic is that of `mimo_oracle.moe_pairs` (engine/mimo_stream/model.py:173-182 for M = 1 and
model.py:221-271 for prefill): per (token, k) pair the gate and up dot products in float64 rounded once
to float32, bf16(g), bf16(u), h = bf16(bf16(g * sig[g]) * u) (kernels.py:79-82 rounding points, the
bf16 sigmoid table of kernels.py:138-146), the down dot product in float64 rounded to float32 and then
to bf16 (gather_qmm returns bf16, model.py:228), and y[t] = bf16(sum over k in order of fp32(out[t, k])
* w[t, k]) with float32 rounding after every product and sum (model.py:266-271).

What differs is only the execution: each distinct expert is dequantised once (e2m1 x e8m0 values are
exact in float32) by torch on all host threads, and all of the expert's pairs go through one float64
matrix product.  With bf16 activations, e2m1 weights and power-of-two scales every dot product here is
exact in float64 (the products' exponents span far less than float64's 53 significant bits), so the
result does not depend on the summation order and equals `mimo_oracle.moe_pairs` bit for bit
(tests/test_oracle.py pins that).  The pool comes as torch CPU tensors in the reference layout
(model.py:32-45), e.g. copied from the device pool under test (whose bytes are pinned to the seeded
generator separately)."""
from __future__ import annotations

from typing import Dict, Optional

import numpy as np
import torch

from . import mimo_oracle as O

# byte -> (even element, odd element): the low nibble holds the even element (kernels.py:19-30)
_BYTE_LUT = torch.tensor(np.stack([O.E2M1[np.arange(256) & 15], O.E2M1[np.arange(256) >> 4]], 1),
                         dtype=torch.float32)
_SIG = None


def _sigtab() -> torch.Tensor:
    global _SIG
    if _SIG is None:
        _SIG = torch.from_numpy(O.sigmoid_table().astype(np.float32))
    return _SIG


def dequant(words: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """MXFP4 words int32/uint32 [out, in/8] + e8m0 uint8 [out, in/32] -> float32 [out, in]
    (element k = nibble k % 8 of word k / 8, low nibble first; kernels.py:19-30)."""
    b = words.contiguous().view(torch.uint8).to(torch.int64)      # little-endian: byte j holds elements 2j, 2j+1
    v = _BYTE_LUT[b].reshape(words.shape[0], -1, 32)              # [out, in/32, 32]
    s = torch.from_numpy(O.e8m0_to_f32(scales.numpy()))           # 2^(s-127), s=0 -> 2^-127, 255 -> NaN
    return (v * s.unsqueeze(-1)).reshape(words.shape[0], -1)


def _bf16(a: torch.Tensor) -> torch.Tensor:
    """float32 -> bf16 (round to nearest even) -> float32."""
    return a.to(torch.bfloat16).to(torch.float32)


def _dots32(Wf: torch.Tensor, X64: torch.Tensor) -> torch.Tensor:
    """X [n, K] . W [N, K]^T in float64 (exact here), rounded once to float32."""
    return (X64 @ Wf.to(torch.float64).T).to(torch.float32)


def swiglu_bf16(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """kernels.py:79-82: gt = bf16(g), ut = bf16(u), h = bf16(bf16(gt * sig[gt]) * ut)."""
    gt = _bf16(g)
    ut = _bf16(u)
    bits = (gt.view(torch.int32) >> 16) & 0xFFFF
    sig = _sigtab()[bits.to(torch.int64)]
    return _bf16(_bf16(gt * sig) * ut)


def expert_outputs(pool: Dict[str, torch.Tensor], slot: int, X: torch.Tensor, round_bf16: bool) -> torch.Tensor:
    """Down outputs [n, H] of the token rows X [n, H] through expert `slot`: fp32(down . h), rounded to
    bf16 when round_bf16 (the gather_qmm pair path, model.py:228), else kept in float32 (kernel B
    before its weight multiply, kernels.py:120)."""
    X64 = X.to(torch.float64)
    g = _dots32(dequant(pool["gate_w"][slot], pool["gate_s"][slot]), X64)
    u = _dots32(dequant(pool["up_w"][slot], pool["up_s"][slot]), X64)
    h = swiglu_bf16(g, u)
    dn = _dots32(dequant(pool["down_w"][slot], pool["down_s"][slot]), h.to(torch.float64))
    return _bf16(dn) if round_bf16 else dn


def pair_outputs(pool: Dict[str, torch.Tensor], slot: int, X: torch.Tensor) -> torch.Tensor:
    """bf16 pair outputs [n, H] (float32 values) of the token rows X [n, H] through expert `slot`."""
    return expert_outputs(pool, slot, X, True)


def _routed(x, pool, inds, w, slot_of, round_bf16: bool, unit_order: bool) -> np.ndarray:
    X = torch.as_tensor(np.asarray(x, np.float32))
    inds = np.asarray(inds)
    T, k = inds.shape
    flat = inds.reshape(-1)
    outs = torch.zeros(T * k, X.shape[1], dtype=torch.float32)
    tok = np.repeat(np.arange(T), k)
    for e in np.unique(flat):
        ps = np.nonzero(flat == e)[0]
        slot = int(e) if slot_of is None else int(slot_of[int(e)])
        outs[torch.from_numpy(ps)] = expert_outputs(pool, slot, X[torch.from_numpy(tok[ps])], round_bf16)
    Y = outs.reshape(T, k, -1)
    wf = torch.as_tensor(np.asarray(w, np.float32))
    order = np.argsort(inds, axis=1, kind="stable") if unit_order else np.broadcast_to(np.arange(k), (T, k))
    rows = torch.arange(T)
    acc = torch.zeros(T, X.shape[1], dtype=torch.float32)
    for j in range(k):
        c = torch.from_numpy(np.ascontiguousarray(order[:, j]))
        acc = acc + Y[rows, c] * wf[rows, c].unsqueeze(1)
    return _bf16(acc).numpy()


def moe_pairs(x, pool: Dict[str, torch.Tensor], inds, w, slot_of: Optional[np.ndarray] = None,
              threads: Optional[int] = None) -> np.ndarray:
    """y [T, H] (float32 values of bf16) of the pair path for token rows x [T, H] (bf16 values) routed
    to inds [T, k] with weights w [T, k]: y[t] = bf16(sum over k in order of fp32(bf16 pair) * w)
    (model.py:173-182, 221-271); `slot_of` maps expert ids to pool slots (default identity)."""
    if threads:
        torch.set_num_threads(threads)
    return _routed(x, pool, inds, w, slot_of, True, False)


def moe_grouped(x, pool: Dict[str, torch.Tensor], inds, w, unit_order: bool = False) -> np.ndarray:
    """The distinct-expert kernels' arithmetic (kernels.py:33-123 + the combine of :194-199):
    part = fp32(down . h) * w in float32, y[t] = bf16(sum of t's parts).  The sum runs in route order
    (gather_idx, kernels.py:198-199) or, with unit_order, in (expert id, row) order - the scatter-add
    of kernels.py:196-197, where a row's routes to distinct experts are met in ascending id order."""
    return _routed(x, pool, inds, w, None, False, unit_order)


def moe_layer(x, pool: Dict[str, torch.Tensor], inds, w) -> np.ndarray:
    """The reference's dispatch rule (model.py:184-219, 324-336): T == 1 or T > 8 -> pair path,
    2 <= T <= 8 -> distinct-expert kernels."""
    T = np.asarray(inds).shape[0]
    return moe_pairs(x, pool, inds, w) if (T == 1 or T > 8) else moe_grouped(x, pool, inds, w)


def pool_to_cpu(pools) -> Dict[str, torch.Tensor]:
    """Host copies of a device pool's six tensors (an ExpertPools object or a dict of tensors)."""
    keys = ("gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")
    return {kk: pools[kk].detach().cpu() for kk in keys}
