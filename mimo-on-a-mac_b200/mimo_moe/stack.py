"""A decode stack of MoE layers: the per-layer loop of the reference engine reduced to its MoE
blocks (engine/mimo_stream/model.py:303-336 runs, per layer, the pre-MoE RMSNorm of model.py:75 and
the MoE block), with the residual stream renormalised between layers:

    y_0 = moe_0(x);  y_l = moe_l(rmsnorm(y_{l-1}))  for l = 1 .. L-1;  returns y_{L-1}

(RMSNorm with unit weight, eps 1e-6).  Each layer's block is the single-GPU `moe_block` or, on N
ranks, the expert-parallel peer exchange with this layer's expert shard (`PeerExpertParallelMoE.layer`,
one set of exchange buffers for all layers).  Every call returns the same output tensor for a given T,
so the whole stack replays as one CUDA graph (`GraphedStep`)."""
from __future__ import annotations

from typing import Callable, Optional, Sequence, Tuple

import torch

from . import ops

Layer = Tuple[torch.Tensor, Optional[torch.Tensor], "ops.ExpertPools"]   # (router W, bias, pools)


class MoEStack:
    """layers: [(router_w bf16 [E, H], bias f32 [E] or None, ExpertPools), ...].

    layer_fn(x, l) -> y replaces the per-layer block (expert parallelism: the peer exchange with
    layer l's weights); the default is the single-GPU block with every expert of layer l resident.
    on_layer(l, x), when set, sees each layer's input (eager runs: route statistics, tests)."""

    def __init__(self, layers: Sequence[Layer], *, eps: float = 1e-6,
                 layer_fn: Optional[Callable[[torch.Tensor, int], torch.Tensor]] = None,
                 status: Optional[torch.Tensor] = None):
        if not layers:
            raise ValueError("empty stack")
        self.layers = list(layers)
        self.eps = eps
        self.status = status
        self.layer_fn = layer_fn
        self.on_layer: Optional[Callable[[int, torch.Tensor], None]] = None
        self._bufs = {}

    def _buffers(self, T: int, H: int, dev):
        key = (T, H, dev)
        if key not in self._bufs:
            self._bufs[key] = tuple(torch.empty(T, H, dtype=torch.bfloat16, device=dev) for _ in range(3))
        return self._bufs[key]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        y_even, y_odd, xn = self._buffers(T, H, x.device)
        y = None
        for li, (W, bias, pools) in enumerate(self.layers):
            if li:
                x = ops.rmsnorm(y, None, self.eps, out=xn)
            if self.on_layer is not None:
                self.on_layer(li, x)
            if self.layer_fn is not None:
                y = self.layer_fn(x, li)
            else:
                y = ops.moe_block(x, W, bias, pools, status=self.status, out=y_odd if li % 2 else y_even)
        return y
