"""Run the reference's own expert-path code on the CPU (TEST INFRASTRUCTURE ONLY).

Uses the artefacts oracle/ref_build.py makes in oracle/_ref/: the reference's Metal kernels A/B
(engine/mimo_stream/kernels.py:33-123) compiled for the CPU, and its numpy group_routes
(kernels.py:149-173).  The final gather + fixed-order sum (kernels.py:198-199) is MLX code; it is
restated here in numpy (float32, summed over k in route order, then bf16).
"""
from __future__ import annotations

import ctypes
import importlib.util
from pathlib import Path

import numpy as np

REF = Path(__file__).resolve().parent / "_ref"
_lib = None
_gr = None


def available() -> bool:
    return (REF / "libref_kernels.so").exists() and (REF / "group_routes_ref.py").exists()


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(REF / "libref_kernels.so"))
        p = ctypes.c_void_p
        L.ref_gateup.argtypes = [ctypes.c_int] * 3 + [p] * 9 + [ctypes.c_int, p]
        L.ref_gateup.restype = ctypes.c_int
        L.ref_down.argtypes = [ctypes.c_int] * 3 + [p] * 6 + [ctypes.c_int, p]
        L.ref_down.restype = ctypes.c_int
        _lib = L
    return _lib


def group_routes(inds, scores, R=8):
    """The reference's own group_routes (kernels.py:149-173), extracted verbatim at build time."""
    global _gr
    if _gr is None:
        spec = importlib.util.spec_from_file_location("group_routes_ref", REF / "group_routes_ref.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _gr = mod.group_routes
    return _gr(np.asarray(inds), np.asarray(scores), R)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def moe_experts(x_bits: np.ndarray, pool: dict, uslot, urows, ucnt, uw, gather_idx, sigtab_bits: np.ndarray,
                R: int = 8):
    """kernels.py:176-199 with kernels A/B executed from the reference's own source.
    x_bits uint16 [M,H] (bf16 bits); pool: dict of numpy arrays in the reference layout, indexed by slot.
    Returns (y_bits uint16 [M,H], h_bits uint16 [U,R,N], part float32 [U,R,H])."""
    x_bits = np.ascontiguousarray(x_bits, np.uint16)
    M, Hd = x_bits.shape
    N = pool["gate_w"].shape[1]
    arr = {k: np.ascontiguousarray(v) for k, v in pool.items()}
    uslot = np.ascontiguousarray(uslot, np.int32)
    urows = np.ascontiguousarray(urows, np.int32)
    ucnt = np.ascontiguousarray(ucnt, np.int32)
    uw = np.ascontiguousarray(uw, np.float32)
    sig = np.ascontiguousarray(sigtab_bits, np.uint16)
    U = uslot.shape[0]
    h = np.zeros((U, R, N), np.uint16)
    part = np.zeros((U, R, Hd), np.float32)
    L = lib()
    rc = L.ref_gateup(R, Hd, N, _p(x_bits), _p(arr["gate_w"]), _p(arr["gate_s"]), _p(arr["up_w"]),
                      _p(arr["up_s"]), _p(uslot), _p(urows), _p(ucnt), _p(sig), U, _p(h))
    if rc != 0:
        raise ValueError(f"ref_gateup: unsupported sizes R={R} K={Hd} N={N}")
    rc = L.ref_down(R, N, Hd, _p(h), _p(arr["down_w"]), _p(arr["down_s"]), _p(uslot), _p(ucnt), _p(uw), U,
                    _p(part))
    if rc != 0:
        raise ValueError(f"ref_down: unsupported sizes R={R} K={N} H={Hd}")
    Y = part.reshape(-1, Hd)[np.asarray(gather_idx, np.int64)].reshape(M, -1, Hd)
    acc = np.zeros((M, Hd), np.float32)
    for j in range(Y.shape[1]):
        acc = (acc + Y[:, j]).astype(np.float32)
    u = acc.view(np.uint32).astype(np.uint64)
    y_bits = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return y_bits, h, part
