"""The reference's MoE-layer path as a vectorised torch CPU program: the timed CPU baseline.

TEST INFRASTRUCTURE ONLY: used by the `cpu_baseline` leg and `--impl reference` arm of `bench.py`, never
by the library.  It restates engine/mimo_stream/model.py:58-65 (router: float32 logits, sigmoid, noaux
bias, top-8, normalised weights) and, per distinct expert, the products of kernels A/B
(engine/mimo_stream/kernels.py:33-123; float32 dot products, bf16 g/u/h roundings) or of the gather_qmm
pair path (model.py:173-182, 221-228; bf16 expert outputs), with the fixed route-order combine
(kernels.py:194-199, model.py:266-271).  Dot products run as float32 torch matrix products on all host
threads, i.e. at the speed a CPU implementation of the path would have, not exactly rounded like
mimo_oracle (which is the checker).

Three variants of the expert weights:
  cached     every needed expert dequantised to float32 before the clock starts (memory permitting:
             13.4 MB of MXFP4 become 100 MB of float32 per expert);
  on the fly the MXFP4 bytes are dequantised inside the timed region, per expert and call;
  native     the packed MXFP4 bytes read directly by a compiled CPU kernel (oracle/cpu_mxfp4.c, built by
             oracle/cpu_port_build.py; AVX2 + FMA where the host has them, OpenMP over output rows).
Time per step = router + sum over the batch's distinct experts + combine; a bounded sample processes
the first experts until the budget is spent and extrapolates by U / done (experts are alike in size).
"""
from __future__ import annotations

import ctypes
import time
from pathlib import Path
from typing import Callable, Dict, Optional

import numpy as np
import torch

from . import batched as B

_NATIVE_LIB = Path(__file__).resolve().with_name("libmimo_cpu_port.so")
_native = None


def native():
    """The compiled CPU kernel (oracle/libmimo_cpu_port.so), or None when it was not built."""
    global _native
    if _native is None and _NATIVE_LIB.exists():
        try:
            L = ctypes.CDLL(str(_NATIVE_LIB))
        except OSError:   # built for another host: the variant is left out
            return None
        p = ctypes.c_void_p
        L.mimo_cpu_port_expert.argtypes = [p, ctypes.c_int, ctypes.c_int, ctypes.c_int, p, p, p, p, p, p,
                                           ctypes.c_int, p, p]
        L.mimo_cpu_port_expert.restype = ctypes.c_int
        L.mimo_cpu_port_isa.restype = ctypes.c_int
        L.mimo_cpu_port_force_scalar.argtypes = [ctypes.c_int]
        L.mimo_cpu_port_set_threads.argtypes = [ctypes.c_int]
        L.mimo_cpu_port_threads.restype = ctypes.c_int
        _native = L
    return _native


def native_expert(raw: Dict[str, torch.Tensor], X: torch.Tensor, pairs: bool) -> torch.Tensor:
    """Expert `raw` (its MXFP4 tensors) on the rows X [R, H] (bf16 values) through the compiled kernel, eight
    rows per call: float32 [R, H] down products (bf16-rounded when pairs)."""
    L = native()
    x = np.ascontiguousarray(X.float().numpy())
    R_all, H = x.shape
    a = {k: np.ascontiguousarray(v.numpy()) for k, v in raw.items()}
    I = a["gate_w"].shape[0]
    out = np.empty((R_all, H), np.float32)
    hbuf = np.empty((8, I), np.float32)
    for r0 in range(0, R_all, 8):
        R = min(8, R_all - r0)
        rc = L.mimo_cpu_port_expert(x[r0:].ctypes.data, R, H, I, a["gate_w"].ctypes.data, a["gate_s"].ctypes.data,
                                    a["up_w"].ctypes.data, a["up_s"].ctypes.data, a["down_w"].ctypes.data,
                                    a["down_s"].ctypes.data, int(pairs), hbuf.ctypes.data, out[r0:].ctypes.data)
        if rc != 0:
            raise ValueError(f"mimo_cpu_port_expert: bad sizes (R={R}, H={H}, I={I})")
    return torch.from_numpy(out)


def _bf16(a: torch.Tensor) -> torch.Tensor:
    return a.to(torch.bfloat16).to(torch.float32)


def route(x: torch.Tensor, W: torch.Tensor, bias: torch.Tensor, k: int = 8):
    """model.py:58-65 in float32: logits, s = sigmoid, sel = s + bias, top-k, w = s / (sum + 1e-20)."""
    logits = x @ W.T
    s = torch.sigmoid(logits)
    _, inds = torch.topk(s + bias, k, dim=-1)
    ws = torch.gather(s, 1, inds)
    return inds, ws / (ws.sum(-1, keepdim=True) + 1e-20)


def _swiglu(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    gt, ut = _bf16(g), _bf16(u)
    return _bf16(_bf16(gt * torch.sigmoid(gt)) * ut)


class CpuLayer:
    """One MoE layer on the host.  `expert(e)` returns expert e's raw MXFP4 tensors as torch CPU tensors
    {gate_w, gate_s, up_w, up_s, down_w, down_s} (reference layout, model.py:32-45)."""

    def __init__(self, W: torch.Tensor, bias: torch.Tensor, expert: Callable[[int], Dict[str, torch.Tensor]]):
        self.W = W.float()
        self.bias = bias.float()
        self.expert = expert

    def step_time(self, x: torch.Tensor, cached: bool, budget_s: float, wall_s: Optional[float] = None,
                  min_experts: int = 2, packed: bool = False, outputs: Optional[list] = None):
        """Seconds of one layer step for the token rows x [T, H] (bf16 values), measured on a bounded
        sample (packed: the compiled kernel on the MXFP4 bytes; else float32 weights, cached or dequantised
        on the fly).  Returns (seconds, experts done, distinct experts U); with `outputs`, appends
        (y, inds, w) of the step it timed (y complete when every expert was done)."""
        xf = x.float()
        T = xf.shape[0]
        t0 = time.perf_counter()
        inds, w = route(xf, self.W, self.bias)
        t_route = time.perf_counter() - t0
        flat = inds.reshape(-1).numpy()
        uids = np.unique(flat)
        pairs = T == 1 or T > 8
        out = torch.zeros(T * inds.shape[1], xf.shape[1])
        wf = w.reshape(-1)
        t_exp, done = 0.0, 0
        wall0 = time.perf_counter()
        for e in uids:
            raw = self.expert(int(e))                    # bytes generated / loaded outside the clock
            ps = torch.from_numpy(np.nonzero(flat == e)[0])
            X = xf[ps // inds.shape[1]]
            if packed:
                t1 = time.perf_counter()
                d = native_expert(raw, X, pairs)
            else:
                if cached:
                    Wg, Wu, Wd = (B.dequant(raw[f"{n}_w"], raw[f"{n}_s"]) for n in ("gate", "up", "down"))
                    t1 = time.perf_counter()
                else:
                    t1 = time.perf_counter()
                    Wg, Wu, Wd = (B.dequant(raw[f"{n}_w"], raw[f"{n}_s"]) for n in ("gate", "up", "down"))
                h = _swiglu(X @ Wg.T, X @ Wu.T)
                d = h @ Wd.T
            out[ps] = (_bf16(d) if pairs else d) * wf[ps].unsqueeze(1)
            t_exp += time.perf_counter() - t1
            done += 1
            if done >= min_experts and (t_exp >= budget_s or (wall_s and time.perf_counter() - wall0 >= wall_s)):
                break
        t2 = time.perf_counter()
        Y = out.reshape(T, inds.shape[1], -1)
        acc = torch.zeros(T, xf.shape[1])
        for j in range(inds.shape[1]):
            acc = acc + Y[:, j]
        y = _bf16(acc)
        t_comb = time.perf_counter() - t2
        if outputs is not None:
            outputs.append((y, inds, w))
        return t_route + t_exp / done * len(uids) + t_comb, done, len(uids)
