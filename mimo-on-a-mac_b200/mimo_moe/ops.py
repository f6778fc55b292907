"""Host interface of the B200 MoE block, mirroring the reference's expert path in engine/mimo_stream.

Reference call surface -> this module:
  Router.__call__            (engine/mimo_stream/model.py:58-65)     -> Router / router()
  group_routes               (engine/mimo_stream/kernels.py:149-173) -> group_routes()
  moe_experts                (engine/mimo_stream/kernels.py:176-199) -> moe_experts()
  Engine._pair_outputs + the combine of Engine._moe_prefill
                             (engine/mimo_stream/model.py:221-271)  -> moe_prefill()
  one MoE layer of Engine.forward, experts resident
                             (engine/mimo_stream/model.py:303-336)  -> moe_block() / MoEBlock

Tensors are torch CUDA tensors; everything runs on the current stream through the C ABI of
libmimo_moe.so.  Outputs are allocated here (caller-side in C terms); scratch comes from a per-device
workspace cache.  Nothing falls back to the CPU.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch

from . import _lib
from ._lib import Pools, check, lib

E_DEFAULT, TOPK, R_DEFAULT = 256, 8, 8
VERIFY_MAX = 8  # model.py:27: T <= 8 uses the small-batch path


@dataclass(frozen=True)
class MoEConfig:
    hidden: int = 4096
    inter: int = 2048
    experts: int = 256
    topk: int = 8
    group: int = 32

    @property
    def expert_bytes(self) -> int:
        return 3 * (self.inter * self.hidden // 2 + self.inter * self.hidden // 32)


# --------------------------------------------------------------------------------------- helpers
def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this library has no CPU path)")


_WS: Dict[int, torch.Tensor] = {}


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Per-device scratch buffer, grown on demand (uint8)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _WS.get(idx)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _WS[idx] = buf
    return buf


def _status(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def read_status(status: torch.Tensor, where: str) -> None:
    """Synchronise on the status word and raise like the reference does for bad routes."""
    code = int(status.item())
    if code == _lib.MIMO_ERANGE:
        raise ValueError(f"{where}: value out of range (expert id, more rows than R routed to one "
                         "expert, or an activation beyond the f16 range)")
    if code != _lib.MIMO_OK:
        raise _lib.MimoError(code, where)


# ------------------------------------------------------------------------------------------ pools
class ExpertPools:
    """One layer's expert pool in the reference layout (model.py:32-45): {gate,up,down}_{w,s}.

    gate_w/up_w [S, I, H/8] 32-bit words, gate_s/up_s [S, I, H/32] uint8, down_w [S, H, I/8],
    down_s [S, H, I/32]."""

    KEYS = ("gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")

    def __init__(self, tensors: Dict[str, torch.Tensor]):
        for k in self.KEYS:
            t = tensors[k]
            _need_cuda(t, k)
            if not t.is_contiguous():
                raise ValueError(f"{k} must be contiguous")
        self.t = {k: tensors[k] for k in self.KEYS}
        gw = self.t["gate_w"]
        self.S, self.inter, self.hidden = gw.shape[0], gw.shape[1], gw.shape[2] * 8
        if tuple(self.t["down_w"].shape) != (self.S, self.hidden, self.inter // 8):
            raise ValueError("down_w shape does not match gate_w")
        self._struct = Pools(*(self.t[k].data_ptr() for k in self.KEYS), self.S, self.hidden, self.inter)

    def __getitem__(self, k):
        return self.t[k]

    @property
    def struct(self) -> Pools:
        return self._struct

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.t.values())

    def slice(self, lo: int, hi: int) -> "ExpertPools":
        """Experts [lo, hi) as a pool of hi - lo slots (views, no copy): one rank's shard."""
        if not 0 <= lo < hi <= self.S:
            raise ValueError(f"bad expert range [{lo}, {hi}) of {self.S}")
        return ExpertPools({k: v[lo:hi] for k, v in self.t.items()})

    @staticmethod
    def empty(S: int, hidden: int = 4096, inter: int = 2048, device=None) -> "ExpertPools":
        device = torch.device(device or "cuda")
        H, I = hidden, inter
        t = {"gate_w": torch.empty(S, I, H // 8, dtype=torch.int32, device=device),
             "gate_s": torch.empty(S, I, H // 32, dtype=torch.uint8, device=device),
             "up_w": torch.empty(S, I, H // 8, dtype=torch.int32, device=device),
             "up_s": torch.empty(S, I, H // 32, dtype=torch.uint8, device=device),
             "down_w": torch.empty(S, H, I // 8, dtype=torch.int32, device=device),
             "down_s": torch.empty(S, H, I // 32, dtype=torch.uint8, device=device)}
        return ExpertPools(t)

    @staticmethod
    def synthetic(S: int = 256, hidden: int = 4096, inter: int = 2048, seed: int = 0, layer: int = 0,
                  first_expert: int = 0, device=None) -> "ExpertPools":
        """Seeded synthetic pool (e2m1 nibbles uniform over 16 codes; scales 2^-7 w.p. 0.6875 else
        2^-8): experts [first_expert, first_expert+S) of `layer` in slots [0, S)."""
        p = ExpertPools.empty(S, hidden, inter, device)
        t = p.t
        check(_lib.testkit().mimo_moe_fill_synthetic_pool(
            t["gate_w"].data_ptr(), t["gate_s"].data_ptr(), t["up_w"].data_ptr(), t["up_s"].data_ptr(),
            t["down_w"].data_ptr(), t["down_s"].data_ptr(), S, hidden, inter, seed, layer, first_expert,
            _stream()), "fill_synthetic_pool")
        return p


# ------------------------------------------------------------------------------------------ router
def router(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, topk: int = TOPK,
           return_logits: bool = False):
    """Router.__call__ (model.py:58-65): FP32 logits, sigmoid, sel = s + bias, top-k (descending sel,
    ties by ascending id), weights = s[idx] / (sum + 1e-20).  Returns (idx int32 [T,k], w fp32 [T,k])."""
    _need_cuda(x, "x")
    x = x.contiguous()
    T, H = x.shape
    E = weight.shape[0]
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("router expects bf16 x and weight")
    logits = torch.empty(T, E, dtype=torch.float32, device=x.device)
    idx = torch.empty(T, topk, dtype=torch.int32, device=x.device)
    w = torch.empty(T, topk, dtype=torch.float32, device=x.device)
    b = None if bias is None else bias.to(device=x.device, dtype=torch.float32).contiguous()
    check(lib().mimo_moe_router(x.data_ptr(), weight.contiguous().data_ptr(), _ptr(b), T, H, E, topk,
                                logits.data_ptr(), idx.data_ptr(), w.data_ptr(), _stream()), "router")
    return (idx, w, logits) if return_logits else (idx, w)


def topk(logits: torch.Tensor, bias: Optional[torch.Tensor] = None, k: int = TOPK):
    """Selection half of the router from given logits (model.py:60-64)."""
    _need_cuda(logits, "logits")
    logits = logits.to(torch.float32).contiguous()
    T, E = logits.shape
    idx = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    b = None if bias is None else bias.to(device=logits.device, dtype=torch.float32).contiguous()
    check(lib().mimo_moe_topk(logits.data_ptr(), _ptr(b), T, E, k, idx.data_ptr(), w.data_ptr(),
                              _stream()), "topk")
    return idx, w


class Router:
    """Drop-in for engine/mimo_stream/model.py:52-65: holds `weight` [E,H] and
    `e_score_correction_bias` [E]; __call__(r) -> (inds [T,k] int32, w [T,k] fp32)."""

    def __init__(self, weight: torch.Tensor, e_score_correction_bias: Optional[torch.Tensor] = None,
                 topk: int = TOPK):
        self.weight = weight.to(torch.bfloat16).contiguous()
        self.e_score_correction_bias = (torch.zeros(weight.shape[0], dtype=torch.float32, device=weight.device)
                                        if e_score_correction_bias is None
                                        else e_score_correction_bias.to(torch.float32).contiguous())
        self.topk = topk

    def __call__(self, r: torch.Tensor):
        r2 = r.reshape(-1, r.shape[-1]).to(torch.bfloat16)
        return router(r2, self.weight, self.e_score_correction_bias, self.topk)


# ------------------------------------------------------------------------------------------ dispatch
@dataclass
class Groups:
    """Output of group_routes (kernels.py:149-173), on the device.  Arrays are sized for
    U_max = min(E, M*k); num_unique[0] holds the live count U."""
    uids: torch.Tensor
    urows: torch.Tensor
    ucnt: torch.Tensor
    uw: torch.Tensor
    gather_idx: torch.Tensor
    num_unique: torch.Tensor
    R: int
    status: torch.Tensor

    def trimmed(self):
        """Host copies trimmed to U (synchronises)."""
        U = int(self.num_unique.item())
        return (self.uids[:U].cpu(), self.urows[:U].cpu(), self.ucnt[:U].cpu(), self.uw[:U].cpu(),
                self.gather_idx.cpu())


def group_routes(inds: torch.Tensor, scores: torch.Tensor, R: int = R_DEFAULT, E: int = E_DEFAULT,
                 check_rows: bool = False) -> Groups:
    """Device grouping of routes by distinct id (kernels.py:149-173).  With check_rows=True this
    synchronises and raises ValueError when more than R rows hit one id, as the reference does."""
    _need_cuda(inds, "inds")
    inds = inds.to(torch.int32).contiguous()
    scores = scores.to(device=inds.device, dtype=torch.float32).contiguous()
    M, k = inds.shape
    ucap = min(E, M * k)
    dev = inds.device
    g = Groups(uids=torch.empty(ucap, dtype=torch.int32, device=dev),
               urows=torch.empty(ucap, R, dtype=torch.int32, device=dev),
               ucnt=torch.empty(ucap, dtype=torch.int32, device=dev),
               uw=torch.empty(ucap, R, dtype=torch.float32, device=dev),
               gather_idx=torch.empty(M * k, dtype=torch.int32, device=dev),
               num_unique=torch.empty(1, dtype=torch.int32, device=dev), R=R, status=_status(dev))
    check(lib().mimo_moe_group_routes(inds.data_ptr(), scores.data_ptr(), M, k, R, E, g.uids.data_ptr(),
                                      g.urows.data_ptr(), g.ucnt.data_ptr(), g.uw.data_ptr(),
                                      g.gather_idx.data_ptr(), g.num_unique.data_ptr(),
                                      g.status.data_ptr(), _stream()), "group_routes")
    if check_rows:
        read_status(g.status, "group_routes")
    return g


def dispatch(inds: torch.Tensor, E: int = E_DEFAULT):
    """Prefill permutation (model.py:235-244, 266-268): (offsets [E+1], order [P], inv [P]) int32."""
    _need_cuda(inds, "inds")
    inds = inds.to(torch.int32).contiguous()
    T, k = inds.shape
    P = T * k
    dev = inds.device
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    order = torch.empty(P, dtype=torch.int32, device=dev)
    inv = torch.empty(P, dtype=torch.int32, device=dev)
    nb = lib().mimo_moe_dispatch_workspace_bytes(T, k, E)
    ws = workspace(nb, dev)
    status = _status(dev)
    check(lib().mimo_moe_dispatch(inds.data_ptr(), T, k, E, offsets.data_ptr(), order.data_ptr(),
                                  inv.data_ptr(), ws.data_ptr(), ws.numel(), status.data_ptr(), _stream()),
          "dispatch")
    return offsets, order, inv


# ------------------------------------------------------------------------------------------ experts
def moe_experts(x: torch.Tensor, pools, uslot: torch.Tensor, urows: torch.Tensor, ucnt: torch.Tensor,
                uw: torch.Tensor, R: int = R_DEFAULT, gather_idx: Optional[torch.Tensor] = None,
                num_unique: Optional[torch.Tensor] = None, pairs_rounding: bool = False,
                status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """kernels.py:176-199: routed expert output for M token rows over distinct experts.
    x bf16 [M,H]; pools: ExpertPools or the reference's dict of tensors; uslot [U] pool slot per
    distinct expert; urows/ucnt/uw from group_routes.  Returns bf16 [M,H]."""
    _need_cuda(x, "x")
    if not isinstance(pools, ExpertPools):
        pools = ExpertPools(pools)
    x = x.to(torch.bfloat16).contiguous()
    M, H = x.shape
    dev = x.device
    uslot = uslot.to(device=dev, dtype=torch.int32).contiguous()
    urows = urows.to(device=dev, dtype=torch.int32).contiguous()
    ucnt = ucnt.to(device=dev, dtype=torch.int32).contiguous()
    uw = uw.to(device=dev, dtype=torch.float32).contiguous()
    U = uslot.shape[0]
    gi = None if gather_idx is None else gather_idx.to(device=dev, dtype=torch.int32).contiguous()
    k = 0 if gi is None else gi.numel() // M
    y = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    nb = lib().mimo_moe_experts_workspace_bytes(M, U, R, pools.hidden, pools.inter)
    ws = workspace(nb, dev)
    st = _status(dev) if status is None else status
    check(lib().mimo_moe_experts(x.data_ptr(), pools.struct, uslot.data_ptr(), urows.data_ptr(),
                                 ucnt.data_ptr(), uw.data_ptr(), _ptr(num_unique), U, R, _ptr(gi), k, M,
                                 int(pairs_rounding), y.data_ptr(), ws.data_ptr(), ws.numel(),
                                 st.data_ptr(), _stream()), "moe_experts")
    return y


def moe_prefill(x: torch.Tensor, pools, inds: torch.Tensor, w: torch.Tensor,
                slot_of: Optional[torch.Tensor] = None, E: Optional[int] = None,
                status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Engine._moe_prefill with every expert resident (model.py:230-271): pairs stable-sorted by expert,
    bf16 pair products, inverse permutation, y = bf16(sum_k fp32(out) * w) in k order."""
    _need_cuda(x, "x")
    if not isinstance(pools, ExpertPools):
        pools = ExpertPools(pools)
    x = x.to(torch.bfloat16).contiguous()
    T, H = x.shape
    dev = x.device
    inds = inds.to(device=dev, dtype=torch.int32).contiguous()
    w = w.to(device=dev, dtype=torch.float32).contiguous()
    k = inds.shape[1]
    so = None if slot_of is None else slot_of.to(device=dev, dtype=torch.int32).contiguous()
    if E is None:
        E = pools.S if so is None else so.numel()
    y = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    nb = lib().mimo_moe_prefill_workspace_bytes(T, k, pools.hidden, pools.inter, E)
    ws = workspace(nb, dev)
    st = _status(dev) if status is None else status
    check(lib().mimo_moe_prefill(x.data_ptr(), pools.struct, _ptr(so), E, inds.data_ptr(), w.data_ptr(),
                                 T, k, y.data_ptr(), ws.data_ptr(), ws.numel(), st.data_ptr(), _stream()),
          "moe_prefill")
    return y


def moe_experts_routes(x: torch.Tensor, pools, idx: torch.Tensor, w: torch.Tensor, expert_base: int = 0,
                       pairs_rounding: bool = False, status: Optional[torch.Tensor] = None,
                       out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-route partials of the routes whose expert is in this pool (experts [expert_base,
    expert_base + S)): float32 [rows * k, H], row r * k + j = fp32(expert products of x[r]) * w[r, j]
    (bf16-rounded products when pairs_rounding), zero for routes to other experts.  The partials of
    all expert shards add exactly (one nonzero term per element), then `combine` sums over k."""
    _need_cuda(x, "x")
    if not isinstance(pools, ExpertPools):
        pools = ExpertPools(pools)
    x = x.to(torch.bfloat16).contiguous()
    rows, H = x.shape
    dev = x.device
    idx = idx.to(device=dev, dtype=torch.int32).contiguous()
    w = w.to(device=dev, dtype=torch.float32).contiguous()
    k = idx.shape[1]
    part = out if out is not None else torch.empty(rows * k, H, dtype=torch.float32, device=dev)
    nb = lib().mimo_moe_experts_routes_workspace_bytes(rows, k, pools.hidden, pools.inter, pools.S)
    ws = workspace(nb, dev)
    st = _status(dev) if status is None else status
    check(lib().mimo_moe_experts_routes(x.data_ptr(), H, rows, pools.struct, expert_base, idx.data_ptr(),
                                        w.data_ptr(), k, k, int(pairs_rounding), part.data_ptr(), None, 0,
                                        ws.data_ptr(), ws.numel(), st.data_ptr(), _stream()), "experts_routes")
    return part


def combine(part: torch.Tensor, M: int, k: int = TOPK, gather_idx: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """kernels.py:194-199: y[m] = bf16(sum over j in order of part[gather_idx[m*k + j]]) (rows m*k + j
    without gather_idx)."""
    _need_cuda(part, "part")
    part = part.to(torch.float32).contiguous()
    H = part.shape[1]
    y = out if out is not None else torch.empty(M, H, dtype=torch.bfloat16, device=part.device)
    gi = None if gather_idx is None else gather_idx.to(device=part.device, dtype=torch.int32).contiguous()
    check(lib().mimo_moe_combine(part.data_ptr(), part.shape[0], _ptr(gi), M, k, H, y.data_ptr(), None, _stream()),
          "combine")
    return y


def rmsnorm(x: torch.Tensor, weight: Optional[torch.Tensor] = None, eps: float = 1e-6,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """model.py:75 (`post_attention_layernorm`, the norm in front of each MoE block):
    y = bf16(x * rsqrt(mean(x^2) + eps)) [* weight], per row, float32 math."""
    _need_cuda(x, "x")
    x = x.to(torch.bfloat16).contiguous()
    T, H = x.shape
    w = None if weight is None else weight.to(device=x.device, dtype=torch.bfloat16).contiguous()
    y = out if out is not None else torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
    check(lib().mimo_moe_rmsnorm(x.data_ptr(), _ptr(w), T, H, float(eps), y.data_ptr(), _stream()), "rmsnorm")
    return y


def combine_pairs(ypair: torch.Tensor, inv: torch.Tensor, w: torch.Tensor, T: int, k: int = TOPK,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """model.py:266-271: y[t] = bf16(sum over j in order of fp32(ypair[inv[t*k + j]]) * w[t, j])."""
    _need_cuda(ypair, "ypair")
    ypair = ypair.to(torch.bfloat16).contiguous()
    inv = inv.to(device=ypair.device, dtype=torch.int32).contiguous()
    w = w.to(device=ypair.device, dtype=torch.float32).contiguous()
    H = ypair.shape[1]
    y = out if out is not None else torch.empty(T, H, dtype=torch.bfloat16, device=ypair.device)
    check(lib().mimo_moe_combine_pairs(ypair.data_ptr(), inv.data_ptr(), w.data_ptr(), T, k, H, y.data_ptr(),
                                       _stream()), "combine_pairs")
    return y


# ------------------------------------------------------------------ expert-parallel prefill exchange
@dataclass
class EpPlan:
    """The send side of one expert-parallel prefill step (mimo_moe_ep_plan): counts [world, 2] int64
    (routes, token rows per destination rank); order / inv [P] (send position <-> route t*k + j);
    send_tok [P] (token of each send row, rows of rank 0 first); send_tag [P, 2] (row within the
    destination's rows, local expert id)."""
    counts: torch.Tensor
    order: torch.Tensor
    inv: torch.Tensor
    send_tok: torch.Tensor
    send_tag: torch.Tensor


def ep_plan(idx: torch.Tensor, per_rank: int, world: int, status: Optional[torch.Tensor] = None) -> EpPlan:
    """Routes of idx [T, k] ordered stably by the rank owning their expert (rank d owns experts
    [d * per_rank, (d + 1) * per_rank)), on the device."""
    _need_cuda(idx, "idx")
    idx = idx.to(torch.int32).contiguous()
    T, k = idx.shape
    P, dev = T * k, idx.device
    counts = torch.empty(world, 2, dtype=torch.int64, device=dev)
    order = torch.empty(P, dtype=torch.int32, device=dev)
    inv = torch.empty(P, dtype=torch.int32, device=dev)
    send_tok = torch.empty(P, dtype=torch.int32, device=dev)
    send_tag = torch.empty(P, 2, dtype=torch.int32, device=dev)
    ws = workspace(lib().mimo_moe_ep_plan_workspace_bytes(T, world), dev)
    st = status if status is not None else _status(dev)
    check(lib().mimo_moe_ep_plan(idx.data_ptr(), T, k, per_rank, world, counts.data_ptr(), order.data_ptr(),
                                 inv.data_ptr(), send_tok.data_ptr(), send_tag.data_ptr(), ws.data_ptr(), ws.numel(),
                                 st.data_ptr(), _stream()), "ep_plan")
    return EpPlan(counts, order, inv, send_tok, send_tag)


def gather_rows(x: torch.Tensor, rows: torch.Tensor, n: int, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[r] = x[rows[r]] for r < n (bf16 rows)."""
    _need_cuda(x, "x")
    x = x.to(torch.bfloat16).contiguous()
    rows = rows.to(device=x.device, dtype=torch.int32).contiguous()
    out = torch.empty(n, x.shape[1], dtype=torch.bfloat16, device=x.device)
    st = status if status is not None else _status(x.device)
    check(lib().mimo_moe_gather_rows(x.data_ptr(), x.shape[0], x.shape[1], rows.data_ptr(), n, out.data_ptr(),
                                     st.data_ptr(), _stream()), "gather_rows")
    return out


def ep_recv_index(recv_tag: torch.Tensor, recv_counts: torch.Tensor, status: Optional[torch.Tensor] = None):
    """Receiving rank: (route_row [n] int32, eid [n] int32), route_row[i] = the index among the received
    rows of the row route i names (its tag's row within the rows from its sender; recv_counts [world, 2]
    = the senders' counts rows), eid[i] = its local expert id."""
    _need_cuda(recv_tag, "recv_tag")
    dev = recv_tag.device
    n = recv_tag.shape[0]
    recv_tag = recv_tag.to(torch.int32).contiguous()
    recv_counts = recv_counts.to(device=dev, dtype=torch.int64).contiguous()
    route_row = torch.empty(n, dtype=torch.int32, device=dev)
    eid = torch.empty(n, dtype=torch.int32, device=dev)
    st = status if status is not None else _status(dev)
    check(lib().mimo_moe_ep_recv_index(recv_tag.data_ptr(), recv_counts.data_ptr(), recv_counts.shape[0], n,
                                       route_row.data_ptr(), eid.data_ptr(), st.data_ptr(), _stream()),
          "ep_recv_index")
    return route_row, eid


def moe_prefill_routes(x: torch.Tensor, pools, route_row: torch.Tensor, eid: torch.Tensor,
                       slot_of: Optional[torch.Tensor] = None, E: Optional[int] = None,
                       status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Per-route prefill products: y[p] = bf16 pair output of expert eid[p] on row route_row[p] of x
    (model.py:221-228), [P, H] bf16."""
    _need_cuda(x, "x")
    if not isinstance(pools, ExpertPools):
        pools = ExpertPools(pools)
    x = x.to(torch.bfloat16).contiguous()
    dev = x.device
    route_row = route_row.to(device=dev, dtype=torch.int32).contiguous()
    eid = eid.to(device=dev, dtype=torch.int32).contiguous()
    P = eid.shape[0]
    so = None if slot_of is None else slot_of.to(device=dev, dtype=torch.int32).contiguous()
    if E is None:
        E = pools.S if so is None else so.numel()
    y = torch.empty(P, pools.hidden, dtype=torch.bfloat16, device=dev)
    ws = workspace(lib().mimo_moe_prefill_workspace_bytes(P, 1, pools.hidden, pools.inter, E), dev)
    st = _status(dev) if status is None else status
    check(lib().mimo_moe_prefill_routes(x.data_ptr(), x.shape[0], pools.struct, _ptr(so), E, route_row.data_ptr(),
                                        eid.data_ptr(), P, y.data_ptr(), ws.data_ptr(), ws.numel(), st.data_ptr(),
                                        _stream()), "moe_prefill_routes")
    return y


def moe_block(x: torch.Tensor, router_w: torch.Tensor, bias: Optional[torch.Tensor], pools,
              topk: int = TOPK, status: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
              return_routes: bool = False):
    """One MoE layer with all experts resident: router, then the reference's dispatch rule
    (model.py:324-336): T == 1 -> stock-path rounding, 2 <= T <= 8 -> distinct-expert kernels,
    T > 8 -> prefill path.  Returns y bf16 [T,H] (and (idx, w) with return_routes)."""
    _need_cuda(x, "x")
    if not isinstance(pools, ExpertPools):
        pools = ExpertPools(pools)
    x = x.to(torch.bfloat16).contiguous()
    T, H = x.shape
    dev = x.device
    E = pools.S
    y = out if out is not None else torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    idx = torch.empty(T, topk, dtype=torch.int32, device=dev) if return_routes else None
    wts = torch.empty(T, topk, dtype=torch.float32, device=dev) if return_routes else None
    b = None if bias is None else bias.to(device=dev, dtype=torch.float32).contiguous()
    nb = lib().mimo_moe_block_workspace_bytes(T, pools.hidden, pools.inter, E, topk)
    ws = workspace(nb, dev)
    st = _status(dev) if status is None else status
    check(lib().mimo_moe_block(x.data_ptr(), router_w.contiguous().data_ptr(), _ptr(b), pools.struct, T,
                               topk, y.data_ptr(), _ptr(idx), _ptr(wts), ws.data_ptr(), ws.numel(),
                               st.data_ptr(), _stream()), "moe_block")
    return (y, idx, wts) if return_routes else y


class MoEBlock:
    """Router + resident expert pool of one layer: __call__(x) -> y (bf16)."""

    def __init__(self, router_weight: torch.Tensor, bias: Optional[torch.Tensor], pools: ExpertPools,
                 topk: int = TOPK):
        self.router_weight = router_weight.to(torch.bfloat16).contiguous()
        self.bias = None if bias is None else bias.to(torch.float32).contiguous()
        self.pools = pools
        self.topk = topk

    def __call__(self, x: torch.Tensor, **kw):
        return moe_block(x, self.router_weight, self.bias, self.pools, self.topk, **kw)
