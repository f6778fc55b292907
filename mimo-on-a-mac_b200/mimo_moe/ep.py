"""Expert parallelism for the MoE block: one process per GPU, experts sharded 256/N per rank.

The reference runs the whole block on one device (engine/mimo_stream/model.py:303-336).  Here rank r
holds experts [r*E/N, (r+1)*E/N) and routes only its own tokens; one step is

  1. route: top-8 of the rank's own T tokens (model.py:58-65), replicated router weights;
  2. dispatch: all-gather of the T token rows and their routes (every rank sees all N*T tokens);
  3. local products: per-route float32 partials of the routes whose expert is local
     (`moe_experts_routes`), zero for every other route;
  4. return: reduce-scatter (sum) of the partials back to the token owners.  Each element has exactly
     one nonzero term, so the sum is exact and does not depend on the collective's order;
  5. combine: the owner adds its tokens' 8 partials in the reference's fixed route order
     (kernels.py:194-199).

Steps 3 and 5 are bit-identical to the single-GPU path, so the block output does not depend on N
(the reference's dispatch rule picks the rounding: T == 1 and T > 8 round each expert's output to
bf16 before the weight, 2 <= T <= 8 keep it in float32).  Every rank must call with the same T.

The compute steps are pluggable (`router_fn`, `experts_fn`, `combine_fn`) so the exchange logic runs
unchanged on CPU `gloo` ranks in the tests, with the CPU oracle as the compute.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import ops

RouterFn = Callable[[torch.Tensor], Tuple[torch.Tensor, torch.Tensor]]


class PhaseTrace:
    """Optional per-phase timing of an eager step: `mark(name)` records a CUDA event on the current
    stream after the work issued since the previous mark; `summary()` gives the mean milliseconds of
    each phase over the recorded steps (call after synchronising).  Never active inside graph capture."""

    def __init__(self):
        self.steps = []

    def start(self):
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self.steps.append([("start", ev)])

    def mark(self, name: str):
        if self.steps:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.steps[-1].append((name, ev))

    def summary(self):
        out = {}
        for marks in self.steps:
            for (_, a), (name, b) in zip(marks, marks[1:]):
                out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        n = max(1, len(self.steps))
        return {k: v / n for k, v in out.items()}
ExpertsFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, bool], torch.Tensor]
CombineFn = Callable[[torch.Tensor, int, int], torch.Tensor]


def expert_range(rank: int, world: int, num_experts: int = 256) -> Tuple[int, int]:
    """Experts owned by `rank`: the contiguous block [rank*E/N, (rank+1)*E/N)."""
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not split over {world} ranks")
    n = num_experts // world
    return rank * n, (rank + 1) * n


def pairs_rounding_for(T: int) -> bool:
    """The reference's dispatch rule (model.py:184-219, 324-336): bf16 expert outputs for T == 1
    (stock gather_qmm path) and T > 8 (prefill pair path); float32 partials for 2 <= T <= 8."""
    return T == 1 or T > 8


class ExpertParallelMoE:
    """One MoE layer over N ranks.  On GPUs the defaults call the CUDA library; `router_fn`,
    `experts_fn`, `combine_fn` replace the compute steps (tests).

    pools_local: this rank's expert shard (slot s = expert expert_base + s);
    router_w / bias: the full router (replicated)."""

    def __init__(self, pools_local, router_w: torch.Tensor, bias: Optional[torch.Tensor], *,
                 num_experts: int = 256, topk: int = 8, group=None, router_fn: Optional[RouterFn] = None,
                 experts_fn: Optional[ExpertsFn] = None, combine_fn: Optional[CombineFn] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.num_experts = num_experts
        self.topk = topk
        self.expert_base, hi = expert_range(self.rank, self.world, num_experts)
        self.pools = pools_local
        if pools_local is not None and getattr(pools_local, "S", hi - self.expert_base) != hi - self.expert_base:
            raise ValueError("local pool does not hold this rank's expert range")
        self.router_w, self.bias = router_w, bias
        self.router_fn = router_fn or (lambda x: ops.router(x, self.router_w, self.bias, topk=self.topk))
        self.experts_fn = experts_fn or (lambda X, I, W, rnd: ops.moe_experts_routes(
            X, self.pools, I, W, expert_base=self.expert_base, pairs_rounding=rnd))
        self.combine_fn = combine_fn or (lambda part, M, k: ops.combine(part, M, k))

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        N, k = self.world, self.topk
        idx, w = self.router_fn(x)
        idx = idx.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        # dispatch: every rank receives all tokens and routes (rank-major order), in one collective
        # over rows packed as [x as int32 words | idx | w bits]
        hw = H * x.element_size() // 4
        row = torch.cat([x.contiguous().view(torch.int32).reshape(T, hw), idx, w.view(torch.int32)], dim=1)
        rows = torch.empty(N * T, hw + 2 * k, dtype=torch.int32, device=x.device)
        dist.all_gather_into_tensor(rows, row, group=self.group)
        X = rows[:, :hw].contiguous().view(x.dtype).reshape(N * T, H)
        IDX = rows[:, hw:hw + k].contiguous()
        W = rows[:, hw + k:].contiguous().view(torch.float32)
        # local per-route partials, zero for other ranks' experts: [N*T*k, H] float32
        part = self.experts_fn(X, IDX, W, pairs_rounding_for(T))
        # return: owner r receives rows [r*T*k, (r+1)*T*k) summed over ranks (one nonzero term each)
        mine = torch.empty(T * k, H, dtype=torch.float32, device=x.device)
        dist.reduce_scatter_tensor(mine, part.contiguous(), op=dist.ReduceOp.SUM, group=self.group)
        return self.combine_fn(mine, T, k)


class GraphedStep:
    """A block for a fixed T captured once as a CUDA graph (collectives included), replayed per step:
    `run(x)` copies x into the graph's input and returns the graph's output tensor (overwritten by
    the next replay).  `block` is any callable x -> y (an expert-parallel block, or the single-GPU
    block with its arguments bound).  Delete the object before destroy_process_group."""

    def __init__(self, block, T: int, H: int, device, dtype=torch.bfloat16, warmup: int = 2):
        self.x = torch.zeros(T, H, dtype=dtype, device=device)
        for _ in range(warmup):  # communicators, tensor maps, workspaces: created outside the capture
            block(self.x)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.y = block(self.x)
        torch.cuda.synchronize(device)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        self.x.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.y


class PeerExpertParallelMoE:
    """Expert parallelism with the exchange inside the kernels, over NVLink peer memory.

    Same steps and results as ExpertParallelMoE (bit-identical to one GPU), without collectives:
      route   `mimo_moe_route_scatter` selects the rank's T tokens' routes and stores each token's
              packed row [x | ids | weights] into every rank's gather buffer (row rank*T + t);
      barrier every rank's rows have landed;
      experts the local experts' products of all N*T tokens; the down kernel stores each route's
              float32 partial straight into its owner's receive buffer (row t*k + j);
      barrier every partial has landed;
      combine fixed route order, from the local receive buffer.
    Two barriers per step also keep a rank from overwriting buffers a peer is still reading.  Buffers
    are plain device allocations shared through CUDA IPC (setup time only); call close() before the
    process group is destroyed.  T is fixed at construction."""

    def __init__(self, pools_local, router_w: torch.Tensor, bias: Optional[torch.Tensor], T: int, *,
                 num_experts: int = 256, topk: int = 8, group=None, timeout_us: int = 0):
        from ._lib import check, lib
        self.timeout_us = timeout_us  # barrier wait limit (0: the library's 2 s)
        self.trace: Optional[PhaseTrace] = None
        self.L, self.check = lib(), check
        self.group = group
        self.world = N = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.T, self.k, self.E = T, topk, num_experts
        self.expert_base, hi = expert_range(self.rank, N, num_experts)
        if pools_local.S != hi - self.expert_base:
            raise ValueError("local pool does not hold this rank's expert range")
        self.pools = pools_local
        self.router_w = router_w.contiguous()
        self.bias = None if bias is None else bias.to(torch.float32).contiguous()
        self.dev = router_w.device
        H = self.H = router_w.shape[1]
        self.ld = H // 2 + 2 * topk  # int32 words per packed row (x rows stay 16-byte aligned)
        sizes = {"rows": N * T * self.ld * 4, "recv": T * topk * H * 4, "sig": 64 * 4}
        self.local, self.opened, ptrs = {}, [], {}
        for name, nbytes in sizes.items():
            p, h = ctypes.c_void_p(), ctypes.create_string_buffer(64)
            check(self.L.mimo_moe_peer_alloc(nbytes, ctypes.addressof(p), ctypes.addressof(h)), "peer_alloc")
            self.local[name] = p.value
            handles = [None] * N
            dist.all_gather_object(handles, h.raw, group=group)
            ptrs[name] = []
            for r, hb in enumerate(handles):
                if r == self.rank:
                    ptrs[name].append(p.value)
                    continue
                q, hbuf = ctypes.c_void_p(), ctypes.create_string_buffer(hb, 64)
                check(self.L.mimo_moe_peer_open(ctypes.addressof(hbuf), ctypes.addressof(q)), "peer_open")
                self.opened.append(q.value)
                ptrs[name].append(q.value)
        self.tab = {n: torch.tensor(v, dtype=torch.int64, device=self.dev) for n, v in ptrs.items()}
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.logits = torch.empty(T, num_experts, dtype=torch.float32, device=self.dev)
        nb = self.L.mimo_moe_experts_routes_workspace_bytes(N * T, topk, H, pools_local.inter, pools_local.S)
        self.ws = torch.empty(nb, dtype=torch.uint8, device=self.dev)
        self.y = torch.empty(T, H, dtype=torch.bfloat16, device=self.dev)
        dist.barrier(group=group)

    def _barrier(self, st: int) -> None:
        self.check(self.L.mimo_moe_peer_barrier(self.tab["sig"].data_ptr(), self.local["sig"], self.rank,
                                                self.world, self.epoch.data_ptr(), self.timeout_us,
                                                self.status.data_ptr(), st),
                   "peer_barrier")

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return self.layer(x, self.pools, self.router_w, self.bias)

    def layer(self, x: torch.Tensor, pools, router_w: torch.Tensor, bias: Optional[torch.Tensor]) -> torch.Tensor:
        """One step with another layer's weights (same shapes) through this object's exchange buffers:
        a stack of layers shares one set of peer buffers.  bias: float32 [E] or None."""
        if tuple(x.shape) != (self.T, self.H):
            raise ValueError(f"x must be [{self.T}, {self.H}]")
        if pools.S != self.pools.S or router_w.shape != self.router_w.shape:
            raise ValueError("layer shapes differ from the exchange's")
        x = x.to(torch.bfloat16).contiguous()
        st = torch.cuda.current_stream(self.dev).cuda_stream
        T, k, H, N = self.T, self.k, self.H, self.world
        tr = self.trace
        if tr:
            tr.start()
        self.check(self.L.mimo_moe_route_scatter(
            x.data_ptr(), T, H, router_w.data_ptr(), None if bias is None else bias.data_ptr(),
            self.E, k, self.tab["rows"].data_ptr(), self.ld, self.rank, N, self.logits.data_ptr(), st),
            "route_scatter")
        if tr:
            tr.mark("route_scatter")
        self._barrier(st)
        if tr:
            tr.mark("barrier_dispatch")
        rows = self.local["rows"]
        self.check(self.L.mimo_moe_experts_routes(
            rows, 2 * self.ld, N * T, pools.struct, self.expert_base, rows + 2 * H,
            rows + 2 * H + 4 * k, self.ld, k, int(pairs_rounding_for(T)), None, self.tab["recv"].data_ptr(),
            T * k, self.ws.data_ptr(), self.ws.numel(), self.status.data_ptr(), st), "experts_routes")
        if tr:
            tr.mark("experts")
        self._barrier(st)
        if tr:
            tr.mark("barrier_return")
        self.check(self.L.mimo_moe_combine(self.local["recv"], T * k, None, T, k, H, self.y.data_ptr(),
                                           self.status.data_ptr(), st), "combine")
        if tr:
            tr.mark("combine")
        return self.y

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after the device is idle)."""
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        for p in self.opened:
            self.L.mimo_moe_peer_close(ctypes.c_void_p(p))
        self.opened = []
        dist.barrier(group=self.group)
        for p in self.local.values():
            self.L.mimo_moe_peer_free(ctypes.c_void_p(p))
        self.local = {}


PairsFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]
CombinePairsFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, int, int], torch.Tensor]
PlanFn = Callable[[torch.Tensor, int, int], "ops.EpPlan"]
GatherFn = Callable[[torch.Tensor, torch.Tensor, int], torch.Tensor]
RecvFn = Callable[[torch.Tensor, torch.Tensor], Tuple[torch.Tensor, torch.Tensor]]


class ExpertParallelPrefill:
    """Expert parallelism for prefill-size batches: routes travel to their expert, not tokens to
    every rank.  One step:

      1. route the rank's own T tokens (model.py:58-65);
      2. plan (mimo_moe_ep_plan, on the device): routes ordered stably by destination rank; each token
         row travels once to every rank that owns one of its experts, with a (row, local expert id) tag
         per route; the counts of routes and rows per destination are exchanged first and cross to the
         host once per step (all-to-all split sizes), then one all-to-all of the rows (gathered by
         mimo_moe_gather_rows) and one of the tags;
      3. expert side: each received route's row among the received token rows (mimo_moe_ep_recv_index),
         then per-route bf16 products straight from those rows (mimo_moe_prefill_routes: each route's
         bf16 pair output, model.py:221-228, the bits the one-GPU prefill combines);
      4. return: the inverse all-to-all;
      5. combine: y[t] = bf16(sum over k in order of fp32(out[t, k]) * w[t, k]) (model.py:266-271).

    Each route's bf16 output is computed by the same kernels as on one GPU, so the result equals the
    single-GPU prefill path bit for bit.  Compute, plan and gather steps are pluggable for the CPU gloo
    tests (which pass torch restatements of the plan and gathers)."""

    def __init__(self, pools_local, router_w: torch.Tensor, bias: Optional[torch.Tensor], *,
                 num_experts: int = 256, topk: int = 8, group=None, router_fn: Optional[RouterFn] = None,
                 pairs_fn: Optional[PairsFn] = None, combine_fn: Optional[CombinePairsFn] = None,
                 plan_fn: Optional[PlanFn] = None, gather_fn: Optional[GatherFn] = None,
                 recv_fn: Optional[RecvFn] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.num_experts, self.topk = num_experts, topk
        self.per_rank = num_experts // self.world
        self.expert_base, _ = expert_range(self.rank, self.world, num_experts)
        self.pools = pools_local
        self.router_w, self.bias = router_w, bias
        self.router_fn = router_fn or (lambda x: ops.router(x, self.router_w, self.bias, topk=self.topk))
        self.pairs_fn = pairs_fn or (lambda rows, rr, e: ops.moe_prefill_routes(rows, self.pools, rr, e,
                                                                                E=self.per_rank))
        self.combine_fn = combine_fn or (lambda yp, inv, w, T, k: ops.combine_pairs(yp, inv, w, T, k))
        self.plan_fn = plan_fn or (lambda idx, per_rank, world: ops.ep_plan(idx, per_rank, world))
        self.gather_fn = gather_fn or (lambda x, rows, n: ops.gather_rows(x, rows, n))
        self.recv_fn = recv_fn or (lambda tag, counts: ops.ep_recv_index(tag, counts))
        self.routes_received = 0  # routes this rank's experts computed, summed over calls
        self.trace: Optional[PhaseTrace] = None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        N, k, dev = self.world, self.topk, x.device
        tr = self.trace
        if tr:
            tr.start()
        if T:
            idx, w = self.router_fn(x)
            idx = idx.to(torch.int32).contiguous()
            w = w.to(torch.float32).contiguous()
            if tr:
                tr.mark("route")
            plan = self.plan_fn(idx, self.per_rank, N)
        else:  # nothing to route; the exchange still runs (the other ranks wait for it)
            w = torch.empty(0, k, dtype=torch.float32, device=dev)
            z = torch.empty(0, dtype=torch.int32, device=dev)
            plan = ops.EpPlan(torch.zeros(N, 2, dtype=torch.int64, device=dev), z, z, z, z.view(0, 2))
        if tr:
            tr.mark("plan")
        recv_counts = torch.empty_like(plan.counts)
        dist.all_to_all_single(recv_counts, plan.counts, group=self.group)
        both = torch.cat([plan.counts, recv_counts]).tolist()  # the step's one host crossing
        if tr:
            tr.mark("counts_exchange")
        sc, rows_sc = [c[0] for c in both[:N]], [c[1] for c in both[:N]]
        rc, rows_rc = [c[0] for c in both[N:]], [c[1] for c in both[N:]]
        self.routes_received += sum(rc)
        send_x = self.gather_fn(x, plan.send_tok, sum(rows_sc)) if T else x[:0]
        send_tag = plan.send_tag[:sum(sc)].contiguous()
        recv_rows = torch.empty(sum(rows_rc), H, dtype=x.dtype, device=dev)
        recv_tag = torch.empty(sum(rc), 2, dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_rows, send_x, rows_rc, rows_sc, group=self.group)
        dist.all_to_all_single(recv_tag, send_tag, rc, sc, group=self.group)
        if tr:
            tr.mark("dispatch_rows")
        if recv_tag.shape[0]:
            route_row, eid = self.recv_fn(recv_tag, recv_counts)
            out = self.pairs_fn(recv_rows, route_row, eid)
        else:
            out = torch.empty(0, H, dtype=x.dtype, device=dev)
        if tr:
            tr.mark("experts")
        back = torch.empty(sum(sc), H, dtype=out.dtype, device=dev)
        dist.all_to_all_single(back, out.contiguous(), sc, rc, group=self.group)
        if tr:
            tr.mark("return_rows")
        y = self.combine_fn(back, plan.inv, w, T, k)
        if tr:
            tr.mark("combine")
        return y
