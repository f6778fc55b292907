"""Torch restatement of the expert-parallel prefill plan and row gathers (the checker for
mimo_moe_ep_plan / mimo_moe_gather_rows / mimo_moe_ep_recv_gather, and the plan the CPU gloo tests
run, where the CUDA library cannot).  Routes p = t*k + j are ordered stably by destination rank
(rank d owns experts [d * per_rank, (d + 1) * per_rank)); within a destination, a token's routes are
adjacent, and the token row travels once to each destination that owns any of its experts."""
import torch

from mimo_moe.ops import EpPlan


def plan(idx: torch.Tensor, per_rank: int, world: int) -> EpPlan:
    idx = idx.to(torch.int32).reshape(idx.shape[0], -1)
    k = idx.shape[1]
    flat = idx.reshape(-1).to(torch.int64)
    P, dev = flat.numel(), flat.device
    dest = flat // per_rank
    order = torch.sort(dest, stable=True).indices                # send position -> route t*k + j
    inv = torch.empty_like(order)
    inv[order] = torch.arange(P, device=dev)                     # route -> send position
    d_s, t_s = dest[order], order // k
    new = torch.ones(P, dtype=torch.bool, device=dev)            # first route of (token, destination)
    if P > 1:
        new[1:] = (d_s[1:] != d_s[:-1]) | (t_s[1:] != t_s[:-1])
    send_counts = torch.bincount(dest, minlength=world)
    row_counts = torch.bincount(d_s[new], minlength=world)
    row_first = torch.cumsum(row_counts, 0) - row_counts
    row_in_seg = (torch.cumsum(new.to(torch.int64), 0) - 1) - row_first[d_s]
    send_tok = torch.zeros(P, dtype=torch.int32, device=dev)
    send_tok[: int(new.sum())] = t_s[new].to(torch.int32)
    send_tag = torch.stack([row_in_seg, flat[order] - d_s * per_rank], 1).to(torch.int32)
    counts = torch.stack([send_counts, row_counts], 1).to(torch.int64)
    return EpPlan(counts, order.to(torch.int32), inv.to(torch.int32), send_tok, send_tag.contiguous())


def gather_rows(x: torch.Tensor, rows: torch.Tensor, n: int) -> torch.Tensor:
    return x[rows[:n].to(torch.int64)].contiguous()


def recv_index(recv_tag: torch.Tensor, recv_counts: torch.Tensor):
    """(row of each received route among the received rows, its local expert id)."""
    rc, rrc = recv_counts[:, 0], recv_counts[:, 1]
    src = torch.repeat_interleave(torch.arange(rc.shape[0], device=rc.device), rc)
    rows = (torch.cumsum(rrc, 0) - rrc)[src] + recv_tag[:, 0].to(torch.int64)
    return rows.to(torch.int32), recv_tag[:, 1].contiguous()
