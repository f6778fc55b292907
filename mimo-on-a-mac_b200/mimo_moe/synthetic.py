"""Seeded synthetic inputs for benchmarks and examples: hidden states, router weights and router
biases, drawn from torch's CPU generator so every process and every box sees the same values.
(Expert pools are filled on the device by `ExpertPools.synthetic`.)

    hidden(T)         x ~ N(0, 1), bf16 [T, H]                      (seed 2)
    router_weight()   W ~ N(0, 0.02), bf16 [E, H]                   (seed 1)
    zipf_bias(c)      bias_e = c * log(p_e * E), p_e ~ Zipf(s) rank weights over a seeded
                      permutation of the experts: skewed expert load  (seed 3)
    overlap_bias()    +beta on a seeded hot subset of experts: consecutive rows share ~2.6 of their
                      8 experts (hot = 22, beta = 0.45, tuned on the seeded decode batches; seed 103)
"""
from __future__ import annotations

import torch


def _gen(seed: int) -> torch.Generator:
    return torch.Generator("cpu").manual_seed(seed)


def hidden(T: int, H: int = 4096, seed: int = 2) -> torch.Tensor:
    return torch.randn(T, H, generator=_gen(seed), dtype=torch.float32).to(torch.bfloat16)


def router_weight(E: int = 256, H: int = 4096, seed: int = 1) -> torch.Tensor:
    return (torch.randn(E, H, generator=_gen(seed), dtype=torch.float32) * 0.02).to(torch.bfloat16)


def zipf_bias(E: int = 256, s: float = 1.1, c: float = 1.0, seed: int = 3) -> torch.Tensor:
    order = torch.randperm(E, generator=_gen(seed))
    rank_of = torch.empty(E, dtype=torch.float64)
    rank_of[order] = torch.arange(1, E + 1, dtype=torch.float64)
    p = rank_of.pow(-s)
    return (c * torch.log(p / p.sum() * E)).to(torch.float32)


def overlap_bias(E: int = 256, hot: int = 22, beta: float = 0.45, seed: int = 3) -> torch.Tensor:
    order = torch.randperm(E, generator=_gen(seed + 100))
    b = torch.zeros(E, dtype=torch.float32)
    b[order[:hot]] = beta
    return b
