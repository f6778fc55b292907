"""Benchmark of the B200 MiMo MoE block (BASELINE.json metric: MoE-layer tok/s + expert HBM GB/s).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload decode8|decode4|decode2|decode1|prefill2048|prefill16384z]
  python bench.py --workload stack48_decode8 [--layers L]   # config 3: a 48-layer decode stack
  python bench.py --impl reference ...     # the reference path's CPU restatement on the host cores

One step = one MoE layer (router -> dispatch -> MXFP4 experts -> combine) over one batch of synthetic
tokens, inputs resident in HBM.  Default workload: BASELINE config 1 at B = 8 rows (decode / MTP
verify), free routing, 256 experts of 13,369,344 B.  Routes rotate over 16 seeded batches, so each step
streams ~0.77 GB of experts chosen from a 3.42 GB pool (inputs > the 126 MB L2).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "mimo-on-a-mac_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

H, I, E, K_TOP = 4096, 2048, 256, 8
EXPERT_BYTES = 3 * (I * H // 2 + I * H // 32)      # 13,369,344
GATEUP_BYTES = 2 * (I * H // 2 + I * H // 32)      # per distinct expert, kernel A
DOWN_BYTES = H * I // 2 + H * I // 32
WORKLOADS = {"decode1": 1, "decode2": 2, "decode4": 4, "decode8": 8, "prefill2048": 2048, "prefill16384z": 16384,
             "stack48_decode1": 1, "stack48_decode8": 8}
STACK_LAYERS = 48  # config 3: 48 MoE layers (~164 GB of experts), RMSNorm (unit weight) between layers
# config 4: Zipf(1.1)-biased routing, bias_e = c * log(p_e * E); c = 0.055 puts the most loaded
# expert at ~10x the mean load on the seeded 16384-token batch (tuned once on the CPU router)
ZIPF_C = 0.055
NBATCH = 16
# DRAM bytes of one decode gate/up launch per distinct expert, from one ncu capture
# (profiles/tc_expert_kernel_decode8_traffic.md): 1.005x the algorithmic 8,912,896
GATEUP_TRAFFIC_PER_EXPERT = 8_957_075


def peaks():
    """(HBM GB/s, sustained dense bf16 TFLOP/s, kind): the driver's measurements, else the pool fallback."""
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    except Exception:
        return 6650.0, 1400.0, "fallback"


def tensor_peaks(dev) -> dict:
    """Dense block-scaled tensor peaks of this GPU measured by the library's own probe
    (mimo_moe_tensor_peak): kind::mxf8f6f4 with e2m1 x e4m3 operands (the expert kernels' MMA form)
    and kind::mxf4 (e2m1 x e2m1, the FP4 rate); best of three 4000-step launches after one warm-up."""
    import ctypes
    import torch
    import mimo_moe
    L = mimo_moe.lib()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    out = {}
    for kind, name in ((0, "mxf8f6f4"), (1, "mxf4")):
        best = 0.0
        for rep in range(4):
            t = ctypes.c_float(0.0)
            _lib_check(L.mimo_moe_tensor_peak(kind, 4000, ctypes.byref(t), status.data_ptr(), stream), "tensor_peak")
            if rep:
                best = max(best, float(t.value))
        out[name] = best
    if int(status.item()) != 0:
        raise RuntimeError(f"device status {int(status.item())} in the tensor peak probe")
    return out


def _lib_check(rc, what):
    from mimo_moe import _lib
    _lib.check(rc, what)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.index)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def make_inputs(B, dev, torch, rank=0):
    from mimo_moe import synthetic
    xs = [synthetic.hidden(B, seed=2 + 1000 * i + 100000 * rank).to(dev) for i in range(NBATCH)]
    W = synthetic.router_weight().to(dev)
    return xs, W


def _host_threads():
    try:
        from threadpoolctl import threadpool_info
        return max([i.get("num_threads", 1) for i in threadpool_info()] + [1])
    except Exception:
        return 1


def cpu_reference_rate(B, budget_s, seed_batch=0):
    """The reference path on the host cores, on a bounded sample of one decode batch of B <= 8 rows:
    the reference's own kernels A/B (engine/mimo_stream/kernels.py:33-123, compiled for the CPU into
    oracle/_ref with OpenMP) and its own group_routes; the router rule (model.py:58-65, MLX on the
    reference's side) and the fixed-order combine restated in numpy.  The batch's distinct experts are
    processed one at a time until `budget_s` is spent (at least one) and the batch time is
    extrapolated by U / k.  Expert bytes are generated before each expert's clock starts.  Without
    oracle/_ref the numpy restatement of the same path is timed instead (kind "port")."""
    import numpy as np
    import torch
    from oracle import mimo_oracle as O
    from oracle import ref_runner as RR
    from oracle import synth
    use_ref = RR.available()
    xt = synth.hidden(B, seed=2 + 1000 * seed_batch)
    x = xt.float().numpy()
    W = synth.router_weight().float().numpy()
    t0 = time.perf_counter()
    _, inds, w = O.router(x, W, np.zeros(E, np.float32))
    uids, urows, ucnt, uw, gidx = (RR.group_routes(inds, w) if use_ref else O.group_routes(inds, w))
    t_fixed = time.perf_counter() - t0
    sp = synth.SynthPool(0, 0)
    sig = O.sigmoid_table_bits() if use_ref else None
    xb = xt.view(torch.int16).numpy().view(np.uint16)
    t_total, done = 0.0, 0
    for u, e in enumerate(uids):
        raw = {n: {int(e): sp[n][int(e)]} for n in ("gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")}
        if use_ref:
            pool = {n: raw[n][int(e)][None] for n in raw}
            one = dict(uslot=np.zeros(1, np.int32), urows=urows[u:u + 1], ucnt=ucnt[u:u + 1], uw=uw[u:u + 1])
            t1 = time.perf_counter()
            RR.moe_experts(xb, pool, one["uslot"], one["urows"], one["ucnt"], one["uw"],
                           np.zeros(B * 8, np.int64), sig)
        else:
            pool = O.Pool(raw, cache=1)
            rows = np.nonzero((inds == e).any(1))[0]
            t1 = time.perf_counter()
            d = pool.deq(int(e))
            h = O.swiglu_bf16(O._dots32(d["gate"], x[rows]), O._dots32(d["up"], x[rows]))
            O._dots32(d["down"], h)
        t_total += time.perf_counter() - t1
        done += 1
        if t_total >= budget_s:
            break
    per_batch = t_fixed + t_total / done * len(uids)
    kind = "reference" if use_ref else "port"
    what = ("the reference's kernels A/B and group_routes (oracle/_ref, OpenMP) + numpy router/combine"
            if use_ref else "numpy restatement of the path")
    return B / per_batch, _host_threads() if not use_ref else int(os.environ.get("OMP_NUM_THREADS", os.cpu_count())), \
        kind, f"{what}: {done} of {len(uids)} distinct experts of one B={B} decode batch, extrapolated by " \
              f"U/k ({t_total:.1f} s of CPU work)"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # all host threads for the OpenMP reference kernels (torchrun sets 1 per process); before loading
    os.environ["OMP_NUM_THREADS"] = str(os.cpu_count() or 1)
    B = WORKLOADS[args.workload]
    budget = max(0.5, min(20.0, 150.0 / max(1, args.steps + args.warmup)))
    rates = []
    for s in range(args.warmup + args.steps):
        r, cores, kind, sample = cpu_reference_rate(min(B, 8), budget, seed_batch=s % NBATCH)
        if s >= args.warmup:
            rates.append(r)
    v = statistics.median(rates)
    metric = f"MoE-layer tok/s ({args.workload})"
    if args.workload.startswith("stack"):  # L layers per token: the one-layer rate / L
        v /= args.layers
        metric = f"MoE-stack tok/s ({args.workload}, {args.layers} layers)"
        sample = f"one layer's rate / {args.layers} layers; {sample}"
    out = {"impl": "reference", "metric": metric, "value": v,
           "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
           "higher_is_better": True, "dtype": "f32 (the reference's kernel code on the CPU)", "data": "synthetic",
           "config": {"workload": args.workload, "B": B, "experts": E, "hidden": H, "inter": I},
           "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample},
           "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out))


def bench_stack(args):
    """one decode step = B tokens per GPU through L MoE layers (RMSNorm, unit weight,
    between layers), experts sharded 256/N per GPU for every layer, the peer-memory exchange per layer
    on N > 1; the whole step replays as one CUDA graph.  Every layer's experts are seeded independently
    (pool layer index l, router W seed 1 + 1000 l, bias 0)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import mimo_moe
    from mimo_moe import _lib, synthetic
    from mimo_moe.ep import GraphedStep, PeerExpertParallelMoE, expert_range
    from mimo_moe.stack import MoEStack

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    B, L = WORKLOADS[args.workload], args.layers
    lo, hi = expert_range(rank, world, E)
    layers = []
    for l in range(L):
        W = synthetic.router_weight(seed=1 + 1000 * l).to(dev)
        pool = mimo_moe.ExpertPools.synthetic(hi - lo, seed=0, layer=l, first_expert=lo, device=dev)
        layers.append((W, None, pool))
    torch.cuda.synchronize()
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    peer = None
    if world > 1:
        peer = PeerExpertParallelMoE(layers[0][2], layers[0][0], None, B, num_experts=E)
        stack = MoEStack(layers, layer_fn=lambda x, l: peer.layer(x, layers[l][2], layers[l][0], None))
    else:
        stack = MoEStack(layers, status=status)
    xs = [synthetic.hidden(B, seed=2 + 1000 * i + 100000 * rank).to(dev) for i in range(NBATCH)]
    gstep = GraphedStep(stack, B, H, dev)
    for i in range(max(3, args.warmup)):
        gstep(xs[i % NBATCH])
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        gstep(xs[i % NBATCH])
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # eager pass: per-launch kernel times, and every layer's routes (all ranks' tokens) per batch ->
    # distinct experts per layer, U (all GPUs) and U_local (this GPU's shard)
    L_ = mimo_moe.lib()
    U, U_local = [], []

    def on_layer(l, x):
        idx, _ = mimo_moe.router(x, layers[l][0], None)
        idx = idx.contiguous()
        if world > 1:
            allidx = torch.empty(world * idx.shape[0], idx.shape[1], dtype=torch.int32, device=dev)
            dist.all_gather_into_tensor(allidx, idx)
            idx = allidx
        u = torch.unique(idx)
        U.append(int(u.numel()))
        U_local.append(int(((u >= lo) & (u < hi)).sum().item()))

    nprof = 4
    _lib.check(L_.mimo_moe_profile_enable(2 * L * nprof + 8), "profile_enable")
    for i in range(nprof):
        stack(xs[i % NBATCH])
    torch.cuda.synchronize()
    launches = (np.zeros(8, np.int32), np.zeros(8, np.float32))
    _lib.check(L_.mimo_moe_profile_read(launches[0].ctypes.data, launches[1].ctypes.data), "profile_read")
    _lib.check(L_.mimo_moe_profile_enable(0), "profile_disable")
    stack.on_layer = on_layer
    for i in range(NBATCH):
        stack(xs[i])
    stack.on_layer = None
    torch.cuda.synchronize()
    st_val = int((peer.status if peer is not None else status).item())
    if st_val != 0:
        raise RuntimeError(f"device status {st_val} during the bench")
    hbm, _, peak_kind = peaks()
    fused = int(launches[0][4]) > 0
    gu_ms = float(launches[1][0]) / max(1, int(launches[0][0]))
    dn_ms = float(launches[1][1]) / max(1, int(launches[0][1]))
    fz_ms = float(launches[1][4]) / max(1, int(launches[0][4]))
    gu_bytes = statistics.mean(U_local) * (EXPERT_BYTES if fused else GATEUP_BYTES)
    achieved = gu_bytes / ((fz_ms if fused else gu_ms) * 1e-3) / 1e9
    step_U = sum(U) / NBATCH                       # distinct experts summed over the L layers, per step
    expert_gbs = step_U * EXPERT_BYTES * args.steps / (ms * 1e-3) / 1e9

    xh = [x.cpu().pin_memory() for x in xs]
    yh = torch.empty(B, H, dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        yd = gstep(xh[i % NBATCH])  # pinned host x straight into the graph's input buffer
        yh.copy_(yd, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r, cores, kind, sample = cpu_reference_rate(B, args.cpu_budget)
        cpu = {"value": r / L, "unit": "tok/s", "cores": cores, "kind": kind,
               "sample": f"one layer's rate / {L} layers; {sample}"}
    if rank == 0:
        tok = B * args.steps * world
        # per layer: single GPU = route (+ memset), gate/up, down, combine; peer exchange = router
        # logits, route+scatter, 2 barriers, unit builder, term split, gate/up, down, combine; plus
        # one RMSNorm between layers
        per_layer = (8 if world > 1 else 4) - (1 if fused else 0)
        out = {
            "metric": f"MoE-stack tok/s ({args.workload}, {L} layers)", "value": tok / (ms * 1e-3), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e2m1 x e4m3 (two-term activations) -> f32, tcgen05 block-scaled",
            "data": "synthetic (48 independently seeded MXFP4 layers, x ~ N(0,1) bf16, router W ~ N(0,0.02))",
            "config": {"workload": args.workload, "layers": L, "B": B * world, "tokens_per_gpu": B,
                       "experts": E, "hidden": H, "inter": I, "topk": K_TOP, "norm": "RMSNorm eps 1e-6, unit weight",
                       "expert_bytes_per_gpu": L * (hi - lo) * EXPERT_BYTES,
                       "mean_distinct_experts_per_layer": statistics.mean(U),
                       "mean_distinct_experts_per_layer_this_gpu": statistics.mean(U_local),
                       "parallelism": (f"ep{world} (experts sharded {E // world} per GPU in every layer; NVLink "
                                       "peer-store exchange per layer, flag barriers)") if world > 1 else "single",
                       "graph": "the whole L-layer step is one CUDA graph",
                       "l2": f"inputs > L2: {L * (hi - lo) * EXPERT_BYTES / 1e9:.1f} GB of experts per GPU"},
            "expert_gbs": expert_gbs,
            "expert_frac_of_measured_hbm": expert_gbs / world / hbm,
            "roofline": {"kernel": "tc_decode_fused_kernel (decode gate/up + SwiGLU + down x weight)" if fused else
                         "tc_expert_kernel<NM=2,NTOK=8,MODE=0> (decode gate/up + SwiGLU)", "bound": "hbm",
                         "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                         "peak_kind": f"{peak_kind} hbm_gbs", "traffic": None,
                         "algorithmic_bytes_per_launch": gu_bytes,
                         "kernel_ms": {"fused": fz_ms} if fused else {"gate_up": gu_ms, "down": dn_ms}},
            "clocks": clk,
            "e2e": {"value": tok / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": B * H * 2,
                    "d2h_bytes_per_step": B * H * 2},
            "gpu_launches": (per_layer * L + (L - 1)) * args.steps,
            "cpu_baseline": cpu,
        }
        print(json.dumps(out))
    del gstep
    torch.cuda.synchronize()
    if peer is not None:
        peer.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode8", choices=list(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--pool-experts", type=int, default=E,
                    help="experts in the pool and router (small cases for profiling; default 256)")
    ap.add_argument("--layers", type=int, default=STACK_LAYERS, help="layers of the stack workloads")
    ap.add_argument("--fixed-batch", type=int, default=None,
                    help="route every step from this one seeded batch (profiling: every captured launch "
                         "then processes the same distinct experts)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload.startswith("stack"):
        return bench_stack(args)

    import numpy as np
    import torch
    import torch.distributed as dist

    import mimo_moe
    from mimo_moe import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    B = WORKLOADS[args.workload]
    NE = args.pool_experts
    ep = world > 1  # expert parallelism: rank r holds experts [r*NE/N, (r+1)*NE/N), routes its own B tokens
    if ep:
        from mimo_moe.ep import expert_range
        lo, hi = expert_range(rank, world, NE)
        pool = mimo_moe.ExpertPools.synthetic(hi - lo, seed=0, layer=0, first_expert=lo, device=dev)
    else:
        lo, hi = 0, NE
        pool = mimo_moe.ExpertPools.synthetic(NE, seed=0, layer=0, device=dev)
    xs, W = make_inputs(B, dev, torch, rank)
    if args.fixed_batch is not None:
        xs = [xs[args.fixed_batch % NBATCH]] * NBATCH
    W = W[:NE].contiguous()
    zipf = args.workload.endswith("z")
    if zipf:
        from mimo_moe import synthetic
        bias = synthetic.zipf_bias(E=NE, c=ZIPF_C).to(dev)
    else:
        bias = torch.zeros(NE, device=dev)
    y = torch.empty(B, H, dtype=torch.bfloat16, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    L = mimo_moe.lib()
    # decode sizes exchange through NVLink peer memory inside the kernels; prefill batches send each
    # route to its expert's rank with NCCL all-to-alls
    peer = ep and B <= 8
    if ep:
        from mimo_moe.ep import ExpertParallelPrefill, PeerExpertParallelMoE
        blk = PeerExpertParallelMoE(pool, W, bias, B, num_experts=NE) if peer else \
            ExpertParallelPrefill(pool, W, bias, num_experts=NE)
    else:
        blk = None
    # expert-parallel decode replays one CUDA graph per step (router, exchanges, expert kernels,
    # combine): the step issues ~8 kernels, whose host-side launch cost would otherwise set the pace.
    # The x copy into the graph's input is inside the step.  The single-GPU decode step (4 kernels + a
    # memset) is replayed as a graph too; prefill steps (whose all-to-all splits are data-dependent)
    # are long enough that launch gaps do not matter and run eagerly.
    from mimo_moe.ep import GraphedStep
    if peer:
        gstep = GraphedStep(blk, B, H, dev)
    elif B <= 8:
        gstep = GraphedStep(lambda x: mimo_moe.moe_block(x, W, bias, pool, status=status, out=y), B, H, dev)
    else:
        gstep = None

    def block(x):
        if gstep is not None:
            return gstep(x)
        return blk(x) if ep else mimo_moe.moe_block(x, W, bias, pool, status=status)

    def step(i):
        if gstep is not None:
            gstep(xs[i % NBATCH])
        elif ep:
            blk(xs[i % NBATCH])
        else:
            mimo_moe.moe_block(xs[i % NBATCH], W, bias, pool, status=status, out=y)

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    _lib.check(L.mimo_moe_profile_enable(4 * args.steps + 8), "profile_enable")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if ep and not peer:
        blk.routes_received = 0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        step(i)
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    # routes this rank's expert kernels computed per step (expert-parallel prefill: skewed routing
    # gives the ranks unequal shares; otherwise each rank computes its own B * k routes)
    routes_step = blk.routes_received / args.steps if ep and not peer else B * K_TOP
    launches = (np.zeros(8, np.int32), np.zeros(8, np.float32))
    _lib.check(L.mimo_moe_profile_read(launches[0].ctypes.data, launches[1].ctypes.data), "profile_read")
    if gstep is not None:  # graph replays carry no profiling events: time the kernels in an eager pass
        nprof = min(args.steps, 50)
        _lib.check(L.mimo_moe_profile_enable(4 * nprof + 8), "profile_enable")
        for i in range(nprof):
            if ep:
                blk(xs[i % NBATCH])
            else:
                mimo_moe.moe_block(xs[i % NBATCH], W, bias, pool, status=status, out=y)
        torch.cuda.synchronize()
        _lib.check(L.mimo_moe_profile_read(launches[0].ctypes.data, launches[1].ctypes.data), "profile_read")
    _lib.check(L.mimo_moe_profile_enable(0), "profile_disable")
    if int(status.item()) != 0:
        raise RuntimeError(f"device status {int(status.item())} during the bench")
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # distinct experts per batch (deterministic routes) -> algorithmic bytes; with expert parallelism
    # U counts the distinct experts over all ranks' tokens (each lives on one rank) and U_local this
    # rank's share, which its kernels stream
    U, U_local = [], []
    for i in range(NBATCH):
        idx, _ = mimo_moe.router(xs[i], W, bias)
        idx = idx.to(torch.int32).contiguous()
        if ep:
            allidx = torch.empty(world * idx.shape[0], idx.shape[1], dtype=torch.int32, device=dev)
            dist.all_gather_into_tensor(allidx, idx)
            idx = allidx
        u = torch.unique(idx)
        U.append(int(u.numel()))
        U_local.append(int(((u >= lo) & (u < hi)).sum().item()))
    steps_U = [U[i % NBATCH] for i in range(args.steps)]
    steps_Ul = [U_local[i % NBATCH] for i in range(args.steps)]
    hbm, tflops_peak, peak_kind = peaks()
    kind_gu, kind_dn = (0, 1) if B <= 8 else (2, 3)
    gu_ms = float(launches[1][kind_gu]) / max(1, int(launches[0][kind_gu]))
    dn_ms = float(launches[1][kind_dn]) / max(1, int(launches[0][kind_dn]))
    fz_ms = float(launches[1][4]) / max(1, int(launches[0][4]))
    gu_bytes = statistics.mean(steps_Ul) * GATEUP_BYTES
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9 if gu_ms > 0 else 0.0
    if B <= 8 and launches[0][4] > 0:  # decode, one launch streams every distinct expert's 3 matrices once
        fz_bytes = statistics.mean(steps_Ul) * EXPERT_BYTES
        fz_gbs = fz_bytes / (fz_ms * 1e-3) / 1e9
        roofline = {"kernel": "tc_decode_fused_kernel (decode gate/up + SwiGLU + down x weight, one launch)",
                    "bound": "hbm", "achieved": fz_gbs, "peak": hbm, "unit": "GB/s", "frac": fz_gbs / hbm,
                    "peak_kind": f"{peak_kind} hbm_gbs", "traffic": None,
                    "algorithmic_bytes_per_launch": fz_bytes}
    elif B <= 8:   # decode: the gate/up kernel streams each distinct expert's gate+up bytes once
        roofline = {"kernel": "tc_expert_kernel<NM=2,NTOK=8,MODE=0> (decode gate/up + SwiGLU)", "bound": "hbm",
                    "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                    "peak_kind": f"{peak_kind} hbm_gbs",
                    "traffic": statistics.mean(steps_Ul) * GATEUP_TRAFFIC_PER_EXPERT,
                    "traffic_source": "ncu dram__bytes_read+write per distinct expert (one capture) x this "
                                      "workload's mean distinct experts",
                    "algorithmic_bytes_per_launch": gu_bytes}
    else:        # prefill: algorithmic FLOPs 2 (gate, up) x 2 x I x H per routed pair
        flops = routes_step * 2 * 2 * I * H
        tf = flops / (gu_ms * 1e-3) / 1e12 if gu_ms > 0 else 0.0
        roofline = {"kernel": "tc_expert_kernel<NM=2,NTOK=64,MODE=0> (prefill gate/up + SwiGLU)", "bound": "tensor",
                    "achieved": tf, "peak": tflops_peak, "unit": "TFLOP/s", "frac": tf / tflops_peak,
                    "peak_kind": f"{peak_kind} bf16_tflops_sustained (dense bf16; the e2m1 x e4m3 MMAs "
                                 "run at the fp8 rate, nominally 2x)",
                    "traffic": None, "algorithmic_flops_per_launch": flops,
                    "weight_gbs": gu_bytes / (gu_ms * 1e-3) / 1e9 if gu_ms > 0 else 0.0}
        # the library's own tcgen05 probe: the MMA form these kernels run (two e4m3 terms per activation,
        # so algorithmic FLOPs are half the executed ones) and the FP4 rate the survey's target names
        tp = tensor_peaks(dev)
        roofline["measured_tensor_tflops"] = tp
        roofline["frac_of_measured_mxf8f6f4"] = tf / tp["mxf8f6f4"] if tp["mxf8f6f4"] > 0 else None
        roofline["frac_of_measured_mxf4"] = tf / tp["mxf4"] if tp["mxf4"] > 0 else None
    roofline["kernel_ms"] = {"fused": fz_ms} if launches[0][4] > 0 else {"gate_up": gu_ms, "down": dn_ms}
    expert_gbs = sum(steps_U) * EXPERT_BYTES / (ms * 1e-3) / 1e9

    # end to end through the public API: pinned host x -> device, block, y -> pinned host
    xh = [x.cpu().pin_memory() for x in xs]
    yh = torch.empty(B, H, dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        if gstep is not None:  # pinned host x straight into the graph's input buffer
            yd = gstep(xh[i % NBATCH])
        else:
            yd = block(xh[i % NBATCH].to(dev, non_blocking=True))
        yh.copy_(yd, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r, cores, kind, sample = cpu_reference_rate(min(B, 8), args.cpu_budget)
        cpu = {"value": r, "unit": "tok/s", "cores": cores, "kind": kind, "sample": sample}

    if rank == 0:
        tok = B * args.steps * world
        # our kernels per step: decode = route (+ its counter memsets, not counted), gate/up + down
        # (one fused launch, or two), combine; prefill = router GEMM, top-k, 3 dispatch, 2 unit
        # builders, term split, gate/up, down, combine
        # expert parallelism, peer exchange: router logits, route+scatter, 2 barriers, unit builder, term
        # split, gate/up, down, combine; all-to-all prefill: router GEMM, top-k, 3 dispatch, 2 unit
        # builders, term split, gate/up, down, per-route combine, weighted combine (the collectives and
        # the route sort / gathers are library kernels)
        fused = int(launches[0][4]) > 0  # decode gate/up + down as one launch
        launches_per_step = ((7 if fused else 8) if peer else 12) if ep else \
            ((3 if fused else 4) if B <= 8 else 11)
        out = {
            "metric": f"MoE-layer tok/s ({args.workload})", "value": tok / (ms * 1e-3), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e2m1 x e4m3 (two-term activations) -> f32, tcgen05 block-scaled",
            "data": "synthetic (seeded MXFP4 pool, x ~ N(0,1) bf16, router W ~ N(0,0.02))",
            "config": {"workload": args.workload, "B": B * world, "experts": NE, "hidden": H, "inter": I,
                       "topk": K_TOP, "routing": f"Zipf(1.1) bias, c={ZIPF_C}" if zipf else "free (bias 0)", "mean_distinct_experts": statistics.mean(steps_U),
                       "mean_distinct_experts_this_gpu": statistics.mean(steps_Ul),
                       "routes_this_gpu_per_step": routes_step,
                       "parallelism": (f"ep{world} (experts sharded {NE // world} per GPU; " +
                                       ("dispatch and return as NVLink peer stores inside the route and "
                                        "down kernels, flag barriers; one CUDA graph per step" if peer else
                                        "NCCL all-to-all of each route to its expert's rank and back") +
                                       "; fixed-order combine)") if ep else "single",
                       "tokens_per_gpu": B,
                       "fixed_batch": args.fixed_batch,
                       "l2": f"inputs > L2: routes rotate over 16 batches of a {NE * EXPERT_BYTES / 1e9:.2f} GB pool"},
            "expert_gbs": expert_gbs,
            "expert_frac_of_measured_hbm": expert_gbs / hbm,
            "roofline": roofline,
            "clocks": clk,
            "e2e": {"value": tok / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": B * H * 2,
                    "d2h_bytes_per_step": B * H * 2},
            "gpu_launches": launches_per_step * args.steps,
            "cpu_baseline": cpu,
        }
        print(json.dumps(out))
    if world > 1:
        del gstep  # a graph holding NCCL calls must be released before the process group
        torch.cuda.synchronize()
        if peer:
            blk.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
