"""Expert files -> HBM pools: the reference's converted checkpoint layout, read into `ExpertPools`.

File format (what scripts/convert-mimo-v26-mlx.py:67-131 writes and engine/mimo_stream/store.py:14-35
reads): one safetensors file per MoE layer, `experts-LNN.safetensors`, holding

    model.layers.{L}.mlp.switch_mlp.{gate,up,down}_proj.weight   U32 [n_experts, out, in/8]
    model.layers.{L}.mlp.switch_mlp.{gate,up,down}_proj.scales   U8  [n_experts, out, in/32]

(the HF MXFP4 bytes verbatim: e2m1 nibbles low first, e8m0 scales), in that order, each tensor
stacked over the experts, so expert e of a tensor is the byte range base + e * stride.  The header
is an 8-byte little-endian length, then compact JSON space-padded so the data section starts on a
16 KiB boundary, and every tensor size is a multiple of 16 KiB.

Loading is one bulk copy per tensor (`mimo_moe_read_file_spans`: reader threads, pinned staging,
O_DIRECT when aligned); an expert-parallel rank reads only its contiguous expert range
[first, first + count).  Router weights come from the dense file (`dense.safetensors`,
`model.layers.{L}.mlp.gate.weight` bf16 [E, H] and `...gate.e_score_correction_bias`, model.py:97-124).
`save_expert_file` writes the same layout (round trips, fixtures, dumping synthetic pools)."""
from __future__ import annotations

import ctypes
import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import numpy as np
import torch

from ._lib import check, lib

ALIGN = 16384          # data section and tensor sizes (the converter's rule)
DIRECT_ALIGN = 4096    # O_DIRECT offsets and sizes
PROJS = (("gate", "gate_proj"), ("up", "up_proj"), ("down", "down_proj"))
DTYPES = {"U32": (np.uint32, 4), "U8": (np.uint8, 1), "BF16": (None, 2), "F32": (np.float32, 4)}


def read_header(path: str) -> Tuple[int, dict]:
    """(absolute offset of the data section, header dict) of a safetensors file."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path}: not a safetensors file")
        n = struct.unpack("<Q", raw)[0]
        if n > 100 << 20:
            raise ValueError(f"{path}: header length {n} is implausible")
        hdr = json.loads(f.read(n))
    return 8 + n, hdr


def tensor_name(layer: int, proj: str, kind: str) -> str:
    return f"model.layers.{layer}.mlp.switch_mlp.{proj}.{'weight' if kind == 'w' else 'scales'}"


@dataclass(frozen=True)
class TensorLoc:
    base: int          # absolute file offset of expert 0
    stride: int        # bytes per expert
    shape: Tuple[int, ...]


class ExpertFile:
    """Index of one layer's expert file: `loc[(key, kind)]` = (base, stride, shape) for key in
    gate/up/down and kind w/s, as ExpertStore computes it (store.py:25-35), after checking names,
    dtypes, shapes and that the ranges lie inside the file."""

    def __init__(self, path: str, layer: int):
        self.path, self.layer = path, layer
        data, hdr = read_header(path)
        size = os.path.getsize(path)
        self.loc: Dict[Tuple[str, str], TensorLoc] = {}
        n_exp = None
        dims = {}
        for key, proj in PROJS:
            for kind, dt in (("w", "U32"), ("s", "U8")):
                name = tensor_name(layer, proj, kind)
                if name not in hdr:
                    raise ValueError(f"{path}: missing {name}")
                t = hdr[name]
                shape = tuple(int(v) for v in t["shape"])
                a, b = (int(v) for v in t["data_offsets"])
                if t["dtype"] != dt or len(shape) != 3:
                    raise ValueError(f"{path}: {name} is {t['dtype']} {shape}, expected {dt} [n_experts, out, in/k]")
                if b - a != int(np.prod(shape)) * DTYPES[dt][1] or data + b > size:
                    raise ValueError(f"{path}: {name} byte range is inconsistent with its shape or the file size")
                n_exp = shape[0] if n_exp is None else n_exp
                if shape[0] != n_exp:
                    raise ValueError(f"{path}: tensors disagree on the expert count")
                self.loc[(key, kind)] = TensorLoc(data + a, (b - a) // n_exp, shape)
            w, s = self.loc[(key, "w")].shape, self.loc[(key, "s")].shape
            if w[1] != s[1] or w[2] * 8 != s[2] * 32:
                raise ValueError(f"{path}: {key} weight {w} and scales {s} do not match (32 values per scale)")
            dims[key] = (w[1], w[2] * 8)            # (out, in)
        self.num_experts = n_exp
        self.inter, self.hidden = dims["gate"]
        if dims["up"] != dims["gate"] or dims["down"] != (self.hidden, self.inter):
            raise ValueError(f"{path}: projection shapes {dims} are not a SwiGLU expert")
        # every expert slice on a 4 KiB boundary: the reader can use O_DIRECT for whole slices
        self.aligned = all(l.base % DIRECT_ALIGN == 0 and l.stride % DIRECT_ALIGN == 0 for l in self.loc.values())

    def spans(self, pools, first: int, count: int):
        """(file offset, bytes, destination pointer) of experts [first, first+count) per pool tensor."""
        if first < 0 or count < 1 or first + count > self.num_experts:
            raise ValueError(f"experts [{first}, {first + count}) outside the file's {self.num_experts}")
        out = []
        for key, _ in PROJS:
            for kind in ("w", "s"):
                l = self.loc[(key, kind)]
                dst = pools[f"{key}_{kind}"]
                if dst.numel() * dst.element_size() != count * l.stride:
                    raise ValueError(f"pool tensor {key}_{kind} does not hold {count} experts of this file")
                out.append((l.base + first * l.stride, count * l.stride, dst.data_ptr()))
        return out


def _read_spans(path: str, spans, device_dst: bool, threads: int, chunk_bytes: int, direct: bool) -> None:
    from ._lib import MIMO_EINVAL
    arr = (ctypes.c_int64 * (3 * len(spans)))()
    for i, (off, n, dst) in enumerate(spans):
        arr[3 * i], arr[3 * i + 1], arr[3 * i + 2] = off, n, dst
    st = torch.cuda.current_stream().cuda_stream if device_dst else None
    code = lib().mimo_moe_read_file_spans(os.fsencode(path), ctypes.addressof(arr), len(spans), threads,
                                          chunk_bytes, int(direct), int(not device_dst), st)
    if code == MIMO_EINVAL:
        raise ValueError(f"read_file_spans({path}): invalid spans or parameters")
    check(code, f"read_file_spans({path})")


def load_expert_pools(path: str, layer: int, first_expert: int = 0, count: Optional[int] = None, device=None,
                      threads: int = 8, chunk_bytes: int = 16 << 20, direct: bool = True):
    """Experts [first_expert, first_expert + count) of `layer` from its expert file into a new device
    pool (slot s = expert first_expert + s): the reference's slot fill (model.py:32-49, store.py:37-47)
    for a pool that holds the whole range at once."""
    from .ops import ExpertPools
    f = ExpertFile(path, layer)
    count = f.num_experts - first_expert if count is None else count
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise ValueError("expert pools live on a CUDA device")
    pools = ExpertPools.empty(count, f.hidden, f.inter, dev)
    with torch.cuda.device(dev):
        _read_spans(path, f.spans(pools.t, first_expert, count), True, threads, chunk_bytes, direct and f.aligned)
    return pools


def read_expert_bytes(path: str, layer: int, first_expert: int, count: int, threads: int = 4) -> Dict[str, np.ndarray]:
    """Host copy of experts [first_expert, first_expert + count) (numpy arrays shaped like the pool
    tensors), through the same native reader; no device involved."""
    f = ExpertFile(path, layer)
    if first_expert < 0 or count < 1 or first_expert + count > f.num_experts:
        raise ValueError("expert range outside the file")
    out, spans = {}, []
    for key, _ in PROJS:
        for kind in ("w", "s"):
            l = f.loc[(key, kind)]
            dt = np.uint32 if kind == "w" else np.uint8
            a = np.empty((count,) + l.shape[1:], dt)
            out[f"{key}_{kind}"] = a
            spans.append((l.base + first_expert * l.stride, count * l.stride, a.ctypes.data))
    _read_spans(path, spans, False, threads, 1 << 20, False)
    return out


def load_router(dense_path: str, layer: int, device=None):
    """(W bf16 [E, H], bias f32 [E]) of `layer` from the dense file (model.py:97-124: the router of an
    MoE layer is model.layers.{L}.mlp.gate.*; the selection bias is e_score_correction_bias)."""
    data, hdr = read_header(dense_path)

    def take(name):
        if name not in hdr:
            raise ValueError(f"{dense_path}: missing {name}")
        t = hdr[name]
        a, b = (int(v) for v in t["data_offsets"])
        with open(dense_path, "rb") as fh:
            fh.seek(data + a)
            raw = fh.read(b - a)
        if len(raw) != b - a:
            raise ValueError(f"{dense_path}: {name} is truncated")
        if t["dtype"] == "BF16":
            return torch.frombuffer(bytearray(raw), dtype=torch.int16).view(torch.bfloat16).reshape(t["shape"])
        if t["dtype"] == "F32":
            return torch.frombuffer(bytearray(raw), dtype=torch.float32).reshape(t["shape"])
        raise ValueError(f"{dense_path}: {name} has dtype {t['dtype']}")

    pre = f"model.layers.{layer}.mlp.gate."
    W = take(pre + "weight").to(torch.bfloat16)
    bias = take(pre + "e_score_correction_bias").to(torch.float32)
    if device is not None:
        W, bias = W.to(device), bias.to(device)
    return W, bias


def save_expert_file(path: str, layer: int, arrays: Dict[str, np.ndarray]) -> int:
    """Write `arrays` ({gate,up,down}_{w,s}: u32 [n, out, in/8] / u8 [n, out, in/32], or an ExpertPools'
    tensors) as experts-LNN.safetensors in the converter's layout (header padded to 16 KiB, tensors in
    gate/up/down, weight/scales order, metadata {"format": "mlx"}).  Returns the data-section offset."""
    tensors = []
    for key, proj in PROJS:
        for kind, dt in (("w", "U32"), ("s", "U8")):
            a = arrays[f"{key}_{kind}"]
            if isinstance(a, torch.Tensor):
                a = a.detach().cpu().numpy()
            a = np.ascontiguousarray(a).view(DTYPES[dt][0])
            tensors.append((tensor_name(layer, proj, kind), dt, a))
    hdr, off = {}, 0
    for name, dt, a in tensors:
        hdr[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
    hdr["__metadata__"] = {"format": "mlx"}
    hj = json.dumps(hdr, separators=(",", ":")).encode()
    hj += b" " * ((-(8 + len(hj))) % ALIGN)
    tmp = path + ".partial"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for _, _, a in tensors:
            f.write(memoryview(a).cast("B"))
    os.replace(tmp, path)
    return 8 + len(hj)
