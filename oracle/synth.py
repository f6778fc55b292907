"""Seeded synthetic inputs for the MoE block, numpy side (TEST INFRASTRUCTURE ONLY).

The CUDA library fills expert pools on the device with the same counter-based generator
(`mimo_moe_fill_synthetic_pool`), so this module can regenerate, bit for bit, any single expert of a
multi-GB device pool and hand it to the oracle.  The generator is the splitmix64 finaliser
(Steele, Lea & Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014) applied to a
per-tensor key plus a Weyl sequence:

    key(seed, layer, tensor) = mix64(seed) ^ ((layer * 8 + tensor + 1) * GOLDEN)
    word64[j]                = mix64(key + (j + 1) * GOLDEN)          (uint64 wrap-around)

Weights: the u32 pool is filled from little-endian word64 (two u32 words each), i.e. every nibble is
uniform over the 16 e2m1 codes.  Scales: byte b of word64[j] is scale byte 8j+b, set to 120 (2^-7) when
that hash byte is < 176 (p = 0.6875) and to 119 (2^-8) otherwise, so the dequantised weights have
std ~= 0.02 and no scale byte is 0 or 255.

Hidden states, router weights and biases are small and come from torch's CPU generator, seeded
(x: seed 2, router W: seed 1, bias draws: seed 3).
"""
from __future__ import annotations

import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
TENSORS = ("gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")
SCALE_HI, SCALE_LO, SCALE_THRESH = 120, 119, 176


def mix64(z):
    z = np.asarray(z, np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def tensor_key(seed: int, layer: int, tensor: int) -> np.uint64:
    with np.errstate(over="ignore"):
        t = np.uint64(layer * 8 + tensor + 1) * GOLDEN
    return np.uint64(mix64(np.uint64(seed)) ^ t)


def words64(key: np.uint64, start: int, count: int) -> np.ndarray:
    j = np.arange(start + 1, start + 1 + count, dtype=np.uint64)
    with np.errstate(over="ignore"):
        return mix64(key + j * GOLDEN)


def expert_tensor(seed: int, layer: int, name: str, expert: int, shape_out_in) -> np.ndarray:
    """One expert's slice of pool tensor `name` ("gate_w", "down_s", ...) in the reference layout."""
    o, i = shape_out_in
    t = TENSORS.index(name)
    key = tensor_key(seed, layer, t)
    if name.endswith("_w"):
        n64 = o * i // 16                           # u64 per expert (8 nibbles per u32, 2 u32 per u64)
        w = words64(key, expert * n64, n64)
        return w.view(np.uint32).reshape(o, i // 8)
    n64 = o * i // 256                              # 8 scale bytes per u64
    w = words64(key, expert * n64, n64)
    b = w.view(np.uint8)
    return np.where(b < SCALE_THRESH, SCALE_HI, SCALE_LO).astype(np.uint8).reshape(o, i // 32)


class SynthPool:
    """Lazy view of a synthetic pool: pool[name][e] regenerates expert e's slice on the CPU."""

    SHAPES = {"gate": (2048, 4096), "up": (2048, 4096), "down": (4096, 2048)}

    def __init__(self, seed: int = 0, layer: int = 0, shapes=None):
        self.seed, self.layer = seed, layer
        self.shapes = dict(shapes or self.SHAPES)

    def __getitem__(self, name):
        proj = name.split("_")[0]
        outer = self

        class _T:
            def __getitem__(self, e):
                return expert_tensor(outer.seed, outer.layer, name, int(e), outer.shapes[proj])
        return _T()


def hidden(T: int, H: int = 4096, seed: int = 2):
    """x ~ N(0,1) as bf16 (torch CPU generator), returned as a torch bf16 tensor."""
    import torch
    g = torch.Generator("cpu").manual_seed(seed)
    return torch.randn(T, H, generator=g, dtype=torch.float32).to(torch.bfloat16)


def router_weight(E: int = 256, H: int = 4096, seed: int = 1):
    """Router W ~ N(0, 0.02) as bf16 (torch CPU generator)."""
    import torch
    g = torch.Generator("cpu").manual_seed(seed)
    return (torch.randn(E, H, generator=g, dtype=torch.float32) * 0.02).to(torch.bfloat16)


def zipf_bias(E: int = 256, s: float = 1.1, c: float = 1.0, seed: int = 3):
    """Config 4: bias_e = c * log(p_e * E) with p_e ~ Zipf(s) rank weights over a seeded permutation."""
    import torch
    g = torch.Generator("cpu").manual_seed(seed)
    perm = torch.randperm(E, generator=g)
    ranks = torch.empty(E, dtype=torch.float64)
    ranks[perm] = torch.arange(1, E + 1, dtype=torch.float64)
    p = ranks ** (-s)
    p = p / p.sum()
    return (c * torch.log(p * E)).to(torch.float32)


def overlap_bias(E: int = 256, hot: int = 22, beta: float = 0.45, seed: int = 3):
    """Config 1 forced-overlap variant: +beta on a seeded hot subset of experts.  hot = 22, beta = 0.45
    were tuned once with this oracle's router on the 16 seeded 8-row decode batches (x seeds 2 + 1000 i,
    router W seed 1): consecutive rows then share 2.57 of their 8 experts on average (the config asks
    for ~2.6), with ~23 distinct experts per batch."""
    import torch
    g = torch.Generator("cpu").manual_seed(seed + 100)
    perm = torch.randperm(E, generator=g)
    b = torch.zeros(E, dtype=torch.float32)
    b[perm[:hot]] = beta
    return b
