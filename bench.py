"""Benchmark of the B200 MiMo MoE block (BASELINE.json metric: MoE-layer tok/s, decode 1-8 rows and prefill
2k, + expert HBM GB/s against the measured peak).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
  python bench.py --workload stack48_decode8 [--layers L]   # config 3: a 48-layer decode stack
  python bench.py --impl reference ...     # the reference path on the host cores (no GPU)

One step = one MoE layer (router -> dispatch -> MXFP4 experts -> combine) over one batch of synthetic
tokens, inputs resident in HBM.  The default run prints ONE JSON line: the headline workload (BASELINE.json
config 1 at B = 8 rows, decode / MTP verify, free routing, 256 experts of 13,369,344 B) and, on one GPU,
nested results under "configs" for the other configurations the metric names: decode1 (config 0),
decode8_overlap (config 1's forced-overlap variant: rows share experts) and prefill2048 (config 2), each
with its own roofline, end-to-end number and CPU baseline.  Decode routes rotate over 16 seeded batches,
so each step streams experts chosen from a 3.42 GB pool (inputs > the 126 MB L2).
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
# workload -> (tokens per GPU, routing)
WORKLOADS = {"decode1": (1, "free"), "decode2": (2, "free"), "decode4": (4, "free"), "decode8": (8, "free"),
             "decode8_overlap": (8, "overlap"), "prefill2048": (2048, "free"), "prefill16384z": (16384, "zipf"),
             "stack48_decode1": (1, "free"), "stack48_decode8": (8, "free"),
             "layer_decode1": (1, "free"), "layer_decode8": (8, "free"), "layer_prefill2048": (2048, "free"),
             "model48_decode1": (1, "free"), "model48_decode8": (8, "free")}
NESTED = ("decode1", "decode8_overlap", "prefill2048")   # measured beside the default headline on one GPU
# the whole decoder layer around the MoE block (attention with a 4096-token context, then the MoE block),
# measured beside the headline too
LAYER_NESTED = ("layer_decode1", "layer_decode8", "layer_prefill2048")
LAYER_CONTEXT = 4096
STACK_LAYERS = 48  # config 3: 48 MoE layers (~164 GB of experts), RMSNorm (unit weight) between layers
# config 4: Zipf(1.1)-biased routing, bias_e = c * log(p_e * E); c = 0.055 puts the most loaded
# expert at ~10x the mean load on the seeded 16384-token batch (tuned once on the CPU router)
ZIPF_C = 0.055
NBATCH = 16
# DRAM bytes of one decode gate/up launch per distinct expert, from an ncu capture of the decode8 workload
# (dram__bytes_read.sum + dram__bytes_write.sum / distinct experts): 1.005x the algorithmic 8,912,896
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
    (mimo_moe_tensor_peak, in the test and benchmark kit): kind::mxf8f6f4 with e2m1 x e4m3 operands (the
    expert kernels' MMA form) and kind::mxf4 (e2m1 x e2m1, the FP4 rate); best of three 4000-step
    launches after one warm-up."""
    import ctypes
    import torch
    from mimo_moe import _lib as mlib
    L = mlib.testkit()
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


# ------------------------------------------------------------------------------------ workloads
def routing_bias(workload: str, NE: int = E):
    """Router bias of a workload (float32 [NE], CPU): free routing, the forced-overlap variant of config 1
    (+beta on a seeded hot subset, so consecutive rows share experts) or config 4's Zipf skew."""
    import torch
    from mimo_moe import synthetic
    routing = WORKLOADS[workload][1]
    if routing == "zipf":
        return synthetic.zipf_bias(E=NE, c=ZIPF_C)
    if routing == "overlap":
        return synthetic.overlap_bias(E=NE)
    return torch.zeros(NE, dtype=torch.float32)


def routing_text(workload: str) -> str:
    return {"free": "free (bias 0)", "overlap": "forced overlap (overlap_bias: +0.45 on 22 seeded experts; ~2.6 of 8 shared by consecutive rows)",
            "zipf": f"Zipf(1.1) bias, c={ZIPF_C}"}[WORKLOADS[workload][1]]


def batches(workload: str, rank: int = 0):
    """The seeded token batches a workload's steps rotate over (bf16, CPU): 16 for decode, 2 for prefill."""
    from mimo_moe import synthetic
    T = WORKLOADS[workload][0]
    n = NBATCH if T <= 8 else 2
    return [synthetic.hidden(T, seed=2 + 1000 * i + 100000 * rank) for i in range(n)]


def workload_config(workload: str, world: int = 1, NE: int = E) -> dict:
    """The workload definition both arms report (the GPU arm adds nothing to it, so the two `config`
    objects are equal)."""
    T = WORKLOADS[workload][0]
    cfg = {"workload": workload, "B": T * world, "tokens_per_gpu": T, "experts": NE, "hidden": H, "inter": I,
           "topk": K_TOP, "routing": routing_text(workload),
           "parallelism": (f"ep{world} (experts sharded {NE // world} per GPU)" if world > 1 else "single"),
           "l2": (f"inputs > L2: routes rotate over {NBATCH} batches of a {NE * EXPERT_BYTES / 1e9:.2f} GB pool"
                  if T <= 8 else f"inputs > L2: every step streams the whole {NE * EXPERT_BYTES / 1e9:.2f} GB pool")}
    if workload.startswith("stack"):
        cfg["layers"] = STACK_LAYERS
    if workload.startswith("model"):
        cfg["layers"] = STACK_LAYERS
        cfg["model"] = ("48 decoder layers (embedding, final norm and lm_head excluded): layer 0 dense MLP "
                        "(16384), layers 1-47 MoE; full attention (4 kv heads) on every sixth layer from 0, "
                        "128-token sliding window with sinks (8 kv heads) elsewhere; 64 q heads x 192, v 128")
        cfg["context"] = LAYER_CONTEXT
    if workload.startswith("layer"):
        cfg["layer"] = ("MoE decoder layer: RMSNorm, full-attention block (64 q heads x 192, 4 kv heads, v 128, "
                        "64 rotary dims, value scale 0.707), residual + RMSNorm, MoE block, residual")
        cfg["context"] = LAYER_CONTEXT if T <= 8 else 0
    return cfg


# ------------------------------------------------------------------------------------ CPU legs
def _cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def _host_cores() -> int:
    return int(os.environ.get("OMP_NUM_THREADS", 0)) or (os.cpu_count() or 1)


def expert_source(device_pool=None, seed: int = 0, layer: int = 0):
    """expert id -> its raw MXFP4 tensors on the host: copied from the device pool under test when one is
    given (fast), else regenerated by the numpy generator (bit-identical bytes); the last 64 are kept."""
    import numpy as np
    import torch
    from oracle import synth
    cache = {}
    sp = synth.SynthPool(seed, layer)

    def get(e):
        if e not in cache:
            if device_pool is not None:
                cache[e] = {n: device_pool[n][e].cpu() for n in ("gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")}
            else:
                cache[e] = {n: torch.from_numpy(np.ascontiguousarray(sp[n][e]).view(
                    np.int32 if n.endswith("_w") else np.uint8)) for n in ("gate_w", "gate_s", "up_w", "up_s",
                                                                          "down_w", "down_s")}
            while len(cache) > 64:
                cache.pop(next(iter(cache)))
        return cache[e]
    return get


def cpu_port_rates(workload: str, budget_s: float, device_pool=None, samples: int = 1):
    """The CPU restatement of the path (oracle/cpu_path.py) on all host threads, in its variants: float32
    torch matrix products with the dequantised experts cached outside the clock or dequantised on the fly,
    and the compiled kernel on the packed MXFP4 bytes (when oracle/libmimo_cpu_port.so was built): tok/s of
    each, median over `samples` batches, each a bounded sample of one step (experts until `budget_s`,
    extrapolated)."""
    import torch
    from mimo_moe import synthetic
    from oracle.cpu_path import CpuLayer, native
    torch.set_num_threads(_host_cores())
    T = WORKLOADS[workload][0]
    layer = CpuLayer(synthetic.router_weight(), routing_bias(workload), expert_source(device_pool))
    xs = batches(workload)
    out = {}
    variants = [("port_fp32_cached", True, False), ("port_on_the_fly", False, False)]
    if native() is not None:
        native().mimo_cpu_port_set_threads(torch.get_num_threads())   # the same threads as the torch forms
        variants.append(("port_mxfp4_native", False, True))
    for name, cached, packed in variants:
        rates, info = [], None
        for s in range(samples):
            sec, done, U = layer.step_time(xs[s % len(xs)], cached, budget_s, wall_s=2 * budget_s, packed=packed)
            rates.append(T / sec)
            info = (done, U)
        out[name] = {"value": statistics.median(rates), "unit": "tok/s", "cores": torch.get_num_threads(),
                     "sample": f"{info[0]} of {info[1]} distinct experts of one {workload} batch, extrapolated "
                               f"by U/done; median of {samples} batch(es)"}
        if packed:
            out[name]["isa"] = "avx2+fma" if native().mimo_cpu_port_isa() == 2 else "scalar"
            out[name]["cores"] = native().mimo_cpu_port_threads()
    return out


def cpu_emulator_rate(B, budget_s, seed_batch=0):
    """The reference's own kernel code on the host cores: its Metal kernels A/B (engine/mimo_stream/
    kernels.py:33-123) compiled for the CPU into oracle/_ref with OpenMP, its own group_routes, and the
    router (model.py:58-65, MLX on the reference's side) and fixed-order combine restated in numpy, on a
    bounded sample of one decode batch of B <= 8 rows.  This build of the Metal bodies is an exactness
    emulator: each 32-lane SIMD-group body runs twice, lane by lane (record, then replay of simd_sum),
    so it is far slower than a CPU implementation would be; it is reported beside the vectorised port,
    not instead of it.  Returns None when oracle/_ref was not built."""
    import numpy as np
    import torch
    from oracle import mimo_oracle as O
    from oracle import ref_runner as RR
    from oracle import synth
    if not RR.available():
        return None
    xt = synth.hidden(B, seed=2 + 1000 * seed_batch)
    x = xt.float().numpy()
    W = synth.router_weight().float().numpy()
    t0 = time.perf_counter()
    _, inds, w = O.router(x, W, np.zeros(E, np.float32))
    uids, urows, ucnt, uw, gidx = RR.group_routes(inds, w)
    t_fixed = time.perf_counter() - t0
    sp = synth.SynthPool(0, 0)
    sig = O.sigmoid_table_bits()
    xb = xt.view(torch.int16).numpy().view(np.uint16)
    t_total, done = 0.0, 0
    for u, e in enumerate(uids):
        pool = {n: sp[n][int(e)][None] for n in ("gate_w", "gate_s", "up_w", "up_s", "down_w", "down_s")}
        one = dict(uslot=np.zeros(1, np.int32), urows=urows[u:u + 1], ucnt=ucnt[u:u + 1], uw=uw[u:u + 1])
        t1 = time.perf_counter()
        RR.moe_experts(xb, pool, one["uslot"], one["urows"], one["ucnt"], one["uw"], np.zeros(B * 8, np.int64), sig)
        t_total += time.perf_counter() - t1
        done += 1
        if t_total >= budget_s:
            break
    per_batch = t_fixed + t_total / done * len(uids)
    return {"value": B / per_batch, "unit": "tok/s", "cores": _host_cores(),
            "sample": f"the reference's kernels A/B (Metal bodies compiled for the CPU, lane-by-lane exactness "
                      f"emulator) + its group_routes: {done} of {len(uids)} distinct experts of one B={B} "
                      f"decode batch, extrapolated by U/k"}


def cpu_baseline(workload: str, budget_s: float, device_pool=None, emulator: bool = False):
    """`cpu_baseline` object of a result: the faster port variant as the value, every variant beside it."""
    rates = cpu_port_rates(workload, budget_s, device_pool)
    T = WORKLOADS[workload][0]
    if emulator and T <= 8:
        em = cpu_emulator_rate(T, budget_s)
        if em is not None:
            rates["reference_kernels_emulated"] = em
    best = max((k for k in rates if k.startswith("port_")), key=lambda k: rates[k]["value"])
    b = rates[best]
    return {"value": b["value"], "unit": "tok/s", "cores": b["cores"], "kind": "port", "cpu_model": _cpu_model(),
            "sample": f"{best}: the reference path restated for the CPU (oracle/cpu_path.py); " + b["sample"],
            "variants": rates}


def cpu_layer_attention_seconds(T: int, context: int, budget_s: float) -> tuple:
    """The attention half of the decoder layer (q/k/v projections, RoPE, attention over the cache, o_proj) as a
    torch-CPU float32 restatement on all host threads, weights converted outside the clock; a bounded sample
    (a slice of the rows and of the heads, scaled up by the fractions timed).  Returns (seconds per step,
    sample text)."""
    import torch
    from mimo_moe.layer import mimo_full_attention
    torch.set_num_threads(_host_cores())
    c = mimo_full_attention()
    g = torch.Generator().manual_seed(7)
    rows = min(T, 128)
    heads = 4 if T > 8 else c.n_heads
    wqkv = torch.randn(c.qkv_width, H, generator=g) * 0.02
    wo = torch.randn(H, c.n_heads * c.v_head_dim, generator=g) * 0.02
    r = torch.randn(rows, H, generator=g)
    nk = context + T
    k = torch.randn(c.n_kv_heads, nk, c.head_dim, generator=g)
    v = torch.randn(c.n_kv_heads, nk, c.v_head_dim, generator=g)
    q = torch.randn(T, heads, c.head_dim, generator=g)
    G = c.n_heads // c.n_kv_heads
    o = torch.randn(rows, c.n_heads * c.v_head_dim, generator=g)
    qpos = torch.arange(context, context + T)
    half = c.rotary_dim // 2
    t_proj = t_attn = 0.0
    n = 0
    while True:
        t0 = time.perf_counter()
        qkv = r @ wqkv.T
        # RoPE on every q and k head's rotary dims (both halves of each pair), the value scale on v
        ang = (torch.arange(rows, dtype=torch.float32)[:, None]
               * torch.pow(c.rope_theta, -torch.arange(half) * 2.0 / c.rotary_dim))[:, None, :]
        cs, sn = torch.cos(ang), torch.sin(ang)
        qk = qkv[:, :(c.n_heads + c.n_kv_heads) * c.head_dim].reshape(rows, -1, c.head_dim)
        x1, x2 = qk[..., :half], qk[..., half:2 * half]
        _ = torch.cat([x1 * cs - x2 * sn, x1 * sn + x2 * cs], -1)
        _ = qkv[:, (c.n_heads + c.n_kv_heads) * c.head_dim:] * 0.707
        _ = o @ wo.T
        t1 = time.perf_counter()
        for h in range(heads):
            s_ = (q[:, h] @ k[h // G].T) * c.scale
            s_ = s_.masked_fill(torch.arange(nk)[None] > qpos[:, None], float("-inf"))
            _ = torch.softmax(s_, -1) @ v[h // G]
        t2 = time.perf_counter()
        t_proj += t1 - t0
        t_attn += t2 - t1
        n += 1
        if t_proj + t_attn >= budget_s / 4 or n >= 20:
            break
    # the projections scale with the rows, the attention with the heads
    sec = t_proj / n * (T / rows) + t_attn / n * (c.n_heads / heads)
    return sec, (f"torch-CPU float32 attention half: {rows} of {T} rows, {heads} of {c.n_heads} heads over "
                 f"{nk} keys, {n} repetitions, scaled to the full step")


def run_reference(args):
    """The reference arm: the reference path on the host cores for the same workload, config and metric.
    The reference's own implementation is MLX on Metal, which does not exist on Linux; its CPU forms here
    are the vectorised restatement (two variants) and the reference's own kernel code compiled for the
    CPU (decode only).  The value is the fastest of them.  Each of up to 8 sampled steps is a bounded
    sample of one step, so any --steps/--warmup finishes in a few minutes."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload.startswith("model"):
        print(json.dumps({"impl": "reference", "unavailable": "the 48-layer decoder stack's CPU path does not fit a "
                          "bounded sample; the reference arm times the one-layer workloads (decode*, prefill*, "
                          "layer_*) and the MoE stack (stack48_*)"}))
        return
    # all host threads (torchrun sets 1 per process); before any library loads its pool
    os.environ["OMP_NUM_THREADS"] = str(os.cpu_count() or 1)
    wl = args.workload if not args.workload.startswith("stack") else args.workload.split("_", 1)[1]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    T = WORKLOADS[wl][0]
    layer = wl.startswith("layer")
    moe_wl = ("decode8" if T == 8 else ("decode1" if T == 1 else "prefill2048")) if layer else wl
    nsamp = max(1, min(args.steps, 2))
    budget = 2.0 * args.cpu_budget / nsamp
    rates = cpu_port_rates(moe_wl, budget, samples=nsamp)
    if T <= 8:
        em = [cpu_emulator_rate(T, budget / 2, seed_batch=s) for s in range(min(nsamp, 2))]
        if em[0] is not None:
            rates["reference_kernels_emulated"] = dict(em[0], value=statistics.median([e["value"] for e in em]))
    best = max(rates, key=lambda k: rates[k]["value"])
    v = rates[best]["value"]
    metric = f"MoE-layer tok/s ({args.workload})"
    sample = rates[best]["sample"]
    if args.workload.startswith("stack"):  # L layers per token: the one-layer rate / L
        v /= args.layers
        metric = f"MoE-stack tok/s ({args.workload}, {args.layers} layers)"
        sample = f"one layer's rate / {args.layers} layers; {sample}"
    if layer:  # the attention half of the layer beside the MoE block, as the GPU arm's cpu_baseline composes it
        t_att, att_sample = cpu_layer_attention_seconds(T, LAYER_CONTEXT if T <= 8 else 0, budget)
        v = T / (T / v + t_att)
        metric = f"decoder-layer tok/s ({args.workload})"
        sample = f"{att_sample}; plus the MoE block's {best} ({sample})"
    cfg = workload_config(args.workload, world)
    out = {"impl": "reference", "metric": metric, "value": v, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": T * world / v * 1e3, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None,
           "dtype": "f32 (the reference path on the CPU)", "data": "synthetic", "config": cfg,
           "cpu_baseline": {"value": v, "unit": "tok/s", "cores": rates[best]["cores"], "cpu_model": _cpu_model(),
                            "kind": "reference" if best == "reference_kernels_emulated" and not layer else "port",
                            "sample": sample if layer else f"{best}: {sample}", "variants": rates},
           "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out))


# ------------------------------------------------------------------------------------ GPU arm
def measure_layer(args, ctx, workload: str, steps: int, warmup: int, cpu_budget: float):
    """The decoder layer around the MoE block (mimo_moe.layer.DecoderLayer, full attention, MoE MLP) at
    decode (T tokens at position LAYER_CONTEXT of a 4096-token cache) or prefill (T tokens from an empty
    cache): device-timed throughput, per-phase times, the step's HBM roofline (decode) and the attention
    kernel's own roofline, end to end through the public API, and a CPU baseline."""
    import numpy as np
    import torch
    import mimo_moe
    from mimo_moe import _lib, synthetic
    from mimo_moe.layer import (DecoderLayer, MoEMLP, add, add_rmsnorm, attention, linear, mimo_full_attention,
                                rope_store, synthetic_attention)
    dev = ctx.dev
    T = WORKLOADS[workload][0]
    decode = T <= 8
    pool = ctx.pool()
    NE = ctx.NE
    W = synthetic.router_weight().to(dev)[:NE].contiguous()
    bias = routing_bias(workload, NE).to(dev)
    cfg = mimo_full_attention(v_scale=0.707)
    attn = synthetic_attention(cfg, seed=4, device=dev)
    layer = DecoderLayer(attn, MoEMLP(W, bias, pool), None, None, eps=1e-5)
    pos0 = LAYER_CONTEXT if decode else 0
    cache = layer.new_cache(LAYER_CONTEXT + 16 if decode else T, max_chunk=T)
    gk = torch.Generator(device=dev).manual_seed(9)
    cache.k.normal_(generator=gk)
    cache.v.normal_(generator=gk)
    xs = [x.to(dev) for x in batches(workload)]
    nb = len(xs)

    def eager(x):
        cache.offset = pos0     # every step is the step at the same position of the same context
        return layer(x, cache)

    gstep = BatchGraphs(eager, xs) if decode else None

    def step(i):
        if gstep is not None:
            gstep(i % nb)
        else:
            eager(xs[i % nb])

    for i in range(max(3, warmup)):
        step(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(ctx.local)
    clocks.start()
    time.sleep(0.3)
    ms = _timed(ctx, steps, step)
    clk = clocks.stop()

    # per-phase device times from an eager pass (CUDA event pairs between the layer's launches)
    names = ["input_norm", "qkv_gemm", "rope_store", "attention", "o_gemm", "add_norm", "moe_block", "add"]
    samples = {n: [] for n in names}
    nprof = 21 if decode else 7
    for i in range(nprof):
        x = xs[i % nb]
        cache.offset = pos0
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
        ev[0].record()
        r = mimo_moe.rmsnorm(x, None, 1e-5); ev[1].record()
        qkv = linear(r, attn.w_qkv); ev[2].record()
        q = rope_store(qkv, cfg, cache, pos0); ev[3].record()
        o = attention(q, cache, cfg, pos0, attn.sinks); ev[4].record()
        a = linear(o.view(T, -1), attn.w_o); ev[5].record()
        h, r2 = add_rmsnorm(x, a, None, 1e-5); ev[6].record()
        y = layer.mlp(r2); ev[7].record()
        add(h, y); ev[8].record()
        torch.cuda.synchronize()
        for j, n in enumerate(names):
            samples[n].append(ev[j].elapsed_time(ev[j + 1]))
    # the median per phase: an eager pass can catch a host stall between two launches in one iteration
    acc = {n: statistics.median(v) for n, v in samples.items()}
    hbm, tflops_peak, peak_kind = peaks()
    attn_w_bytes = (attn.w_qkv.numel() + attn.w_o.numel()) * 2
    keys = pos0 + T
    kv_bytes = cfg.n_kv_heads * keys * (cfg.head_dim + cfg.v_head_dim) * 2
    U = []
    for x in xs:
        idx, _ = mimo_moe.router(x, W, bias)
        U.append(int(torch.unique(idx).numel()))
    Um = statistics.mean(U)
    step_bytes = attn_w_bytes + kv_bytes + Um * EXPERT_BYTES + NE * H * 2
    step_ms = ms / steps
    if decode:
        achieved = step_bytes / (step_ms * 1e-3) / 1e9
        roofline = {"kernel": "whole decoder-layer step (attention weights, KV cache, router, distinct experts)",
                    "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                    "peak_kind": f"{peak_kind} hbm_gbs", "traffic": None,
                    "algorithmic_bytes_per_step": step_bytes,
                    "attention_kernel": {"kernel": "attn_tc_kernel<192,128> with key splits + attn_merge_kernel",
                                         "bytes": kv_bytes, "ms": acc["attention"],
                                         "achieved_gbs": kv_bytes / (acc["attention"] * 1e-3) / 1e9,
                                         "frac": kv_bytes / (acc["attention"] * 1e-3) / 1e9 / hbm}}
    else:
        pairs = T * (T + 1) // 2
        flops = 2 * pairs * cfg.n_heads * (cfg.head_dim + cfg.v_head_dim)
        tf = flops / (acc["attention"] * 1e-3) / 1e12
        roofline = {"kernel": "attn_tc_kernel<192,128> (causal prefill attention, tcgen05 kind::f16, TMEM "
                              "accumulators, float32 softmax)",
                    "bound": "tensor", "achieved": tf, "peak": tflops_peak, "unit": "TFLOP/s",
                    "frac": tf / tflops_peak, "peak_kind": f"{peak_kind} bf16_tflops_sustained",
                    "traffic": None, "algorithmic_flops_per_launch": flops}
    roofline["phases_ms"] = acc

    xh = [x.cpu().pin_memory() for x in xs]
    yh = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty(T, H, dtype=torch.bfloat16, device=dev)

    def e2e_step(i):
        xd.copy_(xh[i % nb], non_blocking=True)
        yh.copy_(eager(xd), non_blocking=True)
    for i in range(3):
        e2e_step(i)
    e2e_ms = _timed(ctx, steps, e2e_step)
    # our launches per step: rmsnorm, rope_store, attention (+ merge when split), add_rmsnorm, add, the two
    # decode projections with their segment sums (prefill projections are cuBLAS), and the MoE block's
    # (decode: route logits, select, gate/up, down, combine; prefill: 11)
    per_step = 5 + (1 + 4 if decode else 0) + (5 if decode else 11)
    res = {
        "metric": f"decoder-layer tok/s ({workload})", "value": T * steps / (ms * 1e-3), "unit": "tok/s",
        "n_gpus": 1, "steps": steps, "warmup": warmup, "ms_per_step": step_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 attention (tcgen05, f32 softmax) + e2m1 x e4m3 MoE (tcgen05)",
        "data": "synthetic (random-init attention weights N(0,0.02), random bf16 KV cache, seeded MXFP4 pool)",
        "config": workload_config(workload, 1, NE), "mean_distinct_experts": Um, "roofline": roofline, "clocks": clk,
        "e2e": {"value": T * steps / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2,
                "how": "eager mimo_moe.layer.DecoderLayer call per step, pinned host x copied in and y read back"},
        "gpu_launches": per_step * steps,
    }
    if not args.no_cpu_baseline:
        moe_rates = cpu_port_rates("decode8" if T == 8 else ("decode1" if T == 1 else "prefill2048"),
                                   cpu_budget, device_pool=pool)
        best = max(moe_rates, key=lambda k: moe_rates[k]["value"])
        t_moe = T / moe_rates[best]["value"]
        t_att, sample = cpu_layer_attention_seconds(T, pos0, cpu_budget)
        res["cpu_baseline"] = {"value": T / (t_moe + t_att), "unit": "tok/s", "cores": _host_cores(), "kind": "port",
                               "cpu_model": _cpu_model(),
                               "sample": f"{sample}; plus the MoE block's {best} ({moe_rates[best]['sample']})"}
    del gstep
    torch.cuda.synchronize()
    return res


class BatchGraphs:
    """One CUDA graph per resident input batch (decode steps are a few short kernels, so a replayed
    graph keeps host launch costs out of the step; capturing one graph per batch keeps the input copy
    into a single graph's input buffer out of it too).  g(i) replays batch i's step and returns its
    output (the block's fixed output buffer)."""

    def __init__(self, fn, xs, warmup: int = 2):
        import torch
        self.graphs, self.out = [], None
        for x in xs:  # tensor maps, workspaces and communicators are created outside the captures
            for _ in range(warmup):
                fn(x)
        torch.cuda.synchronize()
        for x in xs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.out = fn(x)
            self.graphs.append(g)
        torch.cuda.synchronize()

    def __call__(self, i):
        self.graphs[i].replay()
        return self.out


class Ctx:
    """Process-wide state of the GPU arm: ranks, device, the single-GPU expert pool (shared by the
    workloads measured in one run) and the router weight."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=self.dev)
        self.NE = args.pool_experts
        self._pool = None

    def pool(self):
        import mimo_moe
        if self._pool is None:
            if self.world > 1:
                from mimo_moe.ep import expert_range
                lo, hi = expert_range(self.rank, self.world, self.NE)
                self._pool = mimo_moe.ExpertPools.synthetic(hi - lo, seed=0, layer=0, first_expert=lo, device=self.dev)
            else:
                self._pool = mimo_moe.ExpertPools.synthetic(self.NE, seed=0, layer=0, device=self.dev)
        return self._pool

    def range(self):
        if self.world > 1:
            from mimo_moe.ep import expert_range
            return expert_range(self.rank, self.world, self.NE)
        return 0, self.NE


def _timed(ctx, steps, step):
    """Device time (ms) of `steps` calls of step(i), bracketed by barrier + synchronize, max over ranks."""
    import torch
    import torch.distributed as dist
    if ctx.world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(steps):
        step(i)
    ev1.record()
    torch.cuda.synchronize()
    if ctx.world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    if ctx.world > 1:
        t = torch.tensor([ms], device=ctx.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def measure(args, ctx, workload: str, steps: int, warmup: int, cpu_budget: float, emulator: bool):
    """One workload on the GPU arm: device-timed throughput, the dominant kernel's roofline, the
    end-to-end number through the public API and (rank 0, one GPU) the CPU baseline."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import mimo_moe
    from mimo_moe import _lib, synthetic
    from mimo_moe.ep import PhaseTrace

    world, rank, dev, NE = ctx.world, ctx.rank, ctx.dev, ctx.NE
    B = WORKLOADS[workload][0]
    pool = ctx.pool()
    lo, hi = ctx.range()
    W = synthetic.router_weight().to(dev)[:NE].contiguous()
    bias = routing_bias(workload, NE).to(dev)
    xs = [x.to(dev) for x in batches(workload, rank)]
    if args.fixed_batch is not None:
        xs = [xs[args.fixed_batch % len(xs)]] * len(xs)
    nb = len(xs)
    y = torch.empty(B, H, dtype=torch.bfloat16, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    L = mimo_moe.lib()
    ep = world > 1
    peer = ep and B <= 8
    blk = None
    if ep:
        from mimo_moe.ep import ExpertParallelPrefill, PeerExpertParallelMoE
        blk = PeerExpertParallelMoE(pool, W, bias, B, num_experts=NE) if peer else \
            ExpertParallelPrefill(pool, W, bias, num_experts=NE)

    def eager(x, out=None):
        if ep:
            return blk(x)
        return mimo_moe.moe_block(x, W, bias, pool, status=status, out=y if out is None else out)

    # decode steps (4-9 kernels) replay as CUDA graphs, one per resident input batch, so host launch
    # cost does not set the pace; prefill steps are long enough to run eagerly
    gstep = BatchGraphs(eager, xs) if B <= 8 else None

    def step(i):
        if gstep is not None:
            gstep(i % nb)
        else:
            eager(xs[i % nb])

    for i in range(max(3, warmup)):
        step(i)
    torch.cuda.synchronize()
    clocks = ClockSampler(ctx.local)
    clocks.start()
    time.sleep(0.3)
    _lib.check(L.mimo_moe_profile_enable(6 * steps + 8), "profile_enable")
    if ep and not peer:
        blk.routes_received = 0
    ms = _timed(ctx, steps, step)
    clk = clocks.stop()
    routes_step = blk.routes_received / steps if ep and not peer else B * K_TOP
    launches = (np.zeros(8, np.int32), np.zeros(8, np.float32))
    _lib.check(L.mimo_moe_profile_read(launches[0].ctypes.data, launches[1].ctypes.data), "profile_read")
    phases = None
    if gstep is not None or ep:  # graph replays carry no events: time the kernels in an eager pass
        nprof = min(steps, 50 if B <= 8 else 5)
        _lib.check(L.mimo_moe_profile_enable(6 * nprof + 8), "profile_enable")
        if ep:
            blk.trace = PhaseTrace()
        for i in range(nprof):
            eager(xs[i % nb])
        torch.cuda.synchronize()
        if ep:
            phases = blk.trace.summary()
            blk.trace = None
        _lib.check(L.mimo_moe_profile_read(launches[0].ctypes.data, launches[1].ctypes.data), "profile_read")
    _lib.check(L.mimo_moe_profile_enable(0), "profile_disable")
    st_word = int((blk.status if peer else status).item())
    if st_word != 0:
        raise RuntimeError(f"device status {st_word} during the bench ({workload})")

    # distinct experts per batch (deterministic routes) -> algorithmic bytes; with expert parallelism U
    # counts the distinct experts over all ranks' tokens and U_local this rank's share
    U, U_local, shared = [], [], []
    for x in xs:
        idx, _ = mimo_moe.router(x, W, bias)
        idx = idx.to(torch.int32).contiguous()
        if ep:
            allidx = torch.empty(world * idx.shape[0], idx.shape[1], dtype=torch.int32, device=dev)
            dist.all_gather_into_tensor(allidx, idx)
            idx = allidx
        u = torch.unique(idx)
        U.append(int(u.numel()))
        U_local.append(int(((u >= lo) & (u < hi)).sum().item()))
        if 1 < B <= 8:  # experts shared by consecutive rows (config 1's overlap statistic)
            ic = idx.cpu().numpy()
            shared += [len(set(ic[t]) & set(ic[t + 1])) for t in range(ic.shape[0] - 1)]
    steps_U = [U[i % nb] for i in range(steps)]
    steps_Ul = [U_local[i % nb] for i in range(steps)]
    hbm, tflops_peak, peak_kind = peaks()
    kind_gu, kind_dn = (0, 1) if B <= 8 else (2, 3)
    # one-launch decode kinds: 4 (tile-scheduled fused), 5 (stream-K)
    kind_fz = 5 if int(launches[0][5]) > 0 else 4
    n_gu, n_dn, n_fz = int(launches[0][kind_gu]), int(launches[0][kind_dn]), int(launches[0][kind_fz])
    gu_ms = float(launches[1][kind_gu]) / max(1, n_gu)
    dn_ms = float(launches[1][kind_dn]) / max(1, n_dn)
    fz_ms = float(launches[1][kind_fz]) / max(1, n_fz)
    Ul = statistics.mean(steps_Ul)
    gu_bytes = Ul * GATEUP_BYTES
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9 if gu_ms > 0 else 0.0
    if B <= 8 and n_fz > 0:  # decode, one launch streams every distinct expert's 3 matrices once
        fz_bytes = Ul * EXPERT_BYTES
        fz_gbs = fz_bytes / (fz_ms * 1e-3) / 1e9
        name = ("tc_decode_sk_kernel (stream-K decode: gate/up + SwiGLU, then down x weight, one launch)"
                if kind_fz == 5 else "tc_decode_fused_kernel (decode gate/up + SwiGLU + down x weight, one launch)")
        roofline = {"kernel": name, "bound": "hbm", "achieved": fz_gbs, "peak": hbm, "unit": "GB/s",
                    "frac": fz_gbs / hbm, "peak_kind": f"{peak_kind} hbm_gbs",
                    "traffic": None, "algorithmic_bytes_per_launch": fz_bytes}
    elif B <= 8:   # decode: the gate/up kernel streams each distinct expert's gate+up bytes once
        roofline = {"kernel": "tc_expert_kernel<NM=2,NTOK=8,MODE=0> (decode gate/up + SwiGLU)", "bound": "hbm",
                    "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                    "peak_kind": f"{peak_kind} hbm_gbs", "traffic": Ul * GATEUP_TRAFFIC_PER_EXPERT,
                    "traffic_source": "ncu dram__bytes_read+write per distinct expert (one decode8 capture) x this "
                                      "workload's mean distinct experts",
                    "algorithmic_bytes_per_launch": gu_bytes,
                    "down": {"achieved": Ul * DOWN_BYTES / (dn_ms * 1e-3) / 1e9 if dn_ms > 0 else 0.0,
                             "frac": (Ul * DOWN_BYTES / (dn_ms * 1e-3) / 1e9 / hbm) if dn_ms > 0 else 0.0}}
    else:        # prefill: algorithmic FLOPs 2 (gate, up) x 2 x I x H per routed pair
        flops = routes_step * 2 * 2 * I * H
        tf = flops / (gu_ms * 1e-3) / 1e12 if gu_ms > 0 else 0.0
        roofline = {"kernel": "tc_expert_kernel<NM=2,NTOK=64,MODE=0> (prefill gate/up + SwiGLU)", "bound": "tensor",
                    "achieved": tf, "peak": tflops_peak, "unit": "TFLOP/s", "frac": tf / tflops_peak,
                    "peak_kind": f"{peak_kind} bf16_tflops_sustained (dense bf16; the e2m1 x e4m3 MMAs "
                                 "run at the fp8 rate, nominally 2x)",
                    "traffic": None, "algorithmic_flops_per_launch": flops,
                    "weight_gbs": gu_bytes / (gu_ms * 1e-3) / 1e9 if gu_ms > 0 else 0.0}
        tp = tensor_peaks(dev)
        roofline["measured_tensor_tflops"] = tp
        roofline["frac_of_measured_mxf8f6f4"] = tf / tp["mxf8f6f4"] if tp["mxf8f6f4"] > 0 else None
        roofline["frac_of_measured_mxf4"] = tf / tp["mxf4"] if tp["mxf4"] > 0 else None
        # the whole step against its HBM floor: every expert's bytes once
        roofline["step_hbm_floor_ms"] = Ul * EXPERT_BYTES / (hbm * 1e9) * 1e3
    roofline["kernel_ms"] = {"fused": fz_ms} if n_fz > 0 else {"gate_up": gu_ms, "down": dn_ms}
    for kind, name in ((6, "route"), (7, "combine")):  # the decode chain's other launches (single GPU)
        if int(launches[0][kind]) > 0:
            roofline["kernel_ms"][name] = float(launches[1][kind]) / int(launches[0][kind])
    expert_gbs = sum(steps_U) * EXPERT_BYTES / (ms * 1e-3) / 1e9

    # end to end through the public API, as a drop-in caller makes it: every step copies the step's x from
    # pinned host memory to the device, runs the block (eager call) and reads y back to pinned host memory
    xh = [x.cpu().pin_memory() for x in xs]
    yh = torch.empty(B, H, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty(B, H, dtype=torch.bfloat16, device=dev)

    def e2e_step(i):
        xd.copy_(xh[i % nb], non_blocking=True)
        yd = eager(xd)
        yh.copy_(yd, non_blocking=True)
    for i in range(3):
        e2e_step(i)
    e2e_ms = _timed(ctx, steps, e2e_step)
    e2e_graph = None
    if gstep is not None:   # the same with the block replayed as a CUDA graph (pinned x into its input)
        def g_step(i):
            xs[i % nb].copy_(xh[i % nb], non_blocking=True)
            yd = gstep(i % nb)
            yh.copy_(yd, non_blocking=True)
        g_ms = _timed(ctx, steps, g_step)
        e2e_graph = B * world * steps / (g_ms * 1e-3)

    tok = B * steps * world
    # our kernels per step: decode = route (logits, select), gate/up + down (one fused launch, or two),
    # combine; prefill = router GEMM, top-k, 3 dispatch, 2 unit builders, term split, gate/up,
    # down, combine.  Expert parallelism, peer exchange: router logits, route+scatter, 2 barriers, unit
    # builder, term split, gate/up, down, combine; all-to-all prefill: router GEMM, top-k, 3 exchange plan,
    # send-row gather, received-route gather, 3 dispatch, 2 unit builders, term split, gate/up, down,
    # per-route combine, weighted combine.
    fused = n_fz > 0
    # single-GPU decode: route (router logits, top-k select) + the expert launches (stream-K or fused:
    # one; gate/up and down: two) + the combine when it runs as its own launch (the default; when the
    # down kernel's epilogue combines, the profile records no combine launch)
    per_decode = 2 + (1 if fused else 2) + (1 if int(launches[0][7]) > 0 else 0)
    launches_per_step = ((7 if fused else 8) if peer else 17) if ep else (per_decode if B <= 8 else 11)
    res = {
        "metric": f"MoE-layer tok/s ({workload})", "value": tok / (ms * 1e-3), "unit": "tok/s",
        "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms / steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "e2m1 x e4m3 (two-term activations) -> f32, tcgen05 block-scaled",
        "data": "synthetic (seeded MXFP4 pool, x ~ N(0,1) bf16, router W ~ N(0,0.02))",
        "config": workload_config(workload, world, NE),
        "mean_distinct_experts": statistics.mean(steps_U),
        "mean_distinct_experts_this_gpu": Ul,
        "routes_this_gpu_per_step": routes_step,
        "expert_gbs": expert_gbs,
        "expert_frac_of_measured_hbm": expert_gbs / world / hbm,
        "roofline": roofline,
        "clocks": clk,
        "e2e": {"value": tok / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": B * H * 2,
                "d2h_bytes_per_step": B * H * 2,
                "how": "eager public-API call per step (mimo_moe.moe_block, or the expert-parallel block), "
                       "pinned host x copied in and y read back every step"},
        "gpu_launches": launches_per_step * steps,
    }
    if e2e_graph is not None:
        res["e2e"]["value_graph_replay"] = e2e_graph
    if shared:
        res["mean_experts_shared_by_consecutive_rows"] = statistics.mean(shared)
    if args.fixed_batch is not None:
        res["fixed_batch"] = args.fixed_batch
    if phases is not None:
        res["phases_ms"] = phases
        res["phases_how"] = "eager pass, CUDA events between the exchange's steps on this rank (rank 0)"
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(workload, cpu_budget, device_pool=pool, emulator=emulator)
    else:
        res["cpu_baseline"] = None
    del gstep
    torch.cuda.synchronize()
    if blk is not None and peer:
        blk.close()
    return res


def bench_model(args):
    """The decoder stack of a whole MiMo-like model on one GPU: one decode step = B tokens at position 4096
    through 48 decoder layers (attention over each layer's cache, then the dense MLP or the MoE block), the
    step replayed as one CUDA graph.  Random-init bf16 attention and dense weights drawn on the device, the
    MoE layers' pools and routers seeded per layer like the stack workloads, random bf16 KV caches."""
    import torch
    import mimo_moe
    from mimo_moe import synthetic
    from mimo_moe.ep import GraphedStep
    from mimo_moe.layer import (DecoderLayer, DecoderStack, MoEMLP, mimo_full_attention, mimo_sliding_attention,
                                synthetic_attention, synthetic_dense_mlp)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("the model workloads run on one GPU")
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    B, L = WORKLOADS[args.workload][0], args.layers
    layers, routers = [], []
    for l in range(L):
        cfg = mimo_full_attention(v_scale=0.707) if l % 6 == 0 else mimo_sliding_attention(v_scale=0.707)
        attn = synthetic_attention(cfg, seed=100 + l, device=dev, on_device=True)
        if l == 0:
            mlp = synthetic_dense_mlp(inter=16384, seed=99, device=dev, on_device=True)
            routers.append(None)
        else:
            W = synthetic.router_weight(seed=1 + 1000 * l).to(dev)
            mlp = MoEMLP(W, None, mimo_moe.ExpertPools.synthetic(E, seed=0, layer=l, device=dev))
            routers.append(W)
        layers.append(DecoderLayer(attn, mlp, None, None, eps=1e-5))
    stack = DecoderStack(layers, max_len=LAYER_CONTEXT + 16, max_chunk=B)
    g = torch.Generator(device=dev).manual_seed(9)
    for c in stack.caches:
        c.k.normal_(generator=g)
        c.v.normal_(generator=g)
    torch.cuda.synchronize()
    xs = [synthetic.hidden(B, seed=2 + 1000 * i).to(dev) for i in range(NBATCH)]

    def block(x):
        return stack.at(LAYER_CONTEXT)(x)

    gstep = GraphedStep(block, B, H, dev)
    for i in range(max(3, args.warmup)):
        gstep(xs[i % NBATCH])
    torch.cuda.synchronize()
    clocks = ClockSampler(dev.index)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for i in range(args.steps):
        gstep(xs[i % NBATCH])
    ev1.record()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    # one eager pass per batch: every MoE layer's routes -> distinct experts per step (summed over layers)
    U = []

    def tracer(l):
        def f(d):
            idx, _ = mimo_moe.router(d["r2"], routers[l], None)
            U.append(int(torch.unique(idx).numel()))
        return f
    for l, layer in enumerate(layers):
        layer.trace = tracer(l) if routers[l] is not None else None
    for i in range(NBATCH):
        block(xs[i])
    for layer in layers:
        layer.trace = None
    for layer in layers[1:]:
        layer.mlp.check_status()
    torch.cuda.synchronize()
    hbm, _, peak_kind = peaks()
    attn_bytes = sum((l.attn.w_qkv.numel() + l.attn.w_o.numel()) * 2 for l in layers)
    kv_bytes = sum(c.n_kv_heads * ((min(LAYER_CONTEXT + B, c.window + B - 1) if c.window else LAYER_CONTEXT + B)
                                   * (c.head_dim + c.v_head_dim) * 2) for c in (l.attn.cfg for l in layers))
    dense_bytes = (layers[0].mlp.w_gate_up.numel() + layers[0].mlp.w_down.numel()) * 2
    step_U = sum(U) / NBATCH
    step_bytes = attn_bytes + kv_bytes + dense_bytes + step_U * EXPERT_BYTES + (L - 1) * E * H * 2
    step_ms = ms / args.steps
    achieved = step_bytes / (step_ms * 1e-3) / 1e9

    xh = [x.cpu().pin_memory() for x in xs]
    yh = torch.empty(B, H, dtype=torch.bfloat16).pin_memory()
    xd = torch.empty(B, H, dtype=torch.bfloat16, device=dev)
    e2e_steps = max(3, min(args.steps, 40))

    def e2e_step(i):
        xd.copy_(xh[i % NBATCH], non_blocking=True)
        yh.copy_(block(xd), non_blocking=True)
    e2e_step(0)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(e2e_steps):
        e2e_step(i)
    t1.record()
    torch.cuda.synchronize()
    e2e_ms = t0.elapsed_time(t1)

    def g_step(i):
        xd.copy_(xh[i % NBATCH], non_blocking=True)
        yh.copy_(gstep(xd), non_blocking=True)
    t0.record()
    for i in range(args.steps):
        g_step(i)
    t1.record()
    torch.cuda.synchronize()
    g_ms = t0.elapsed_time(t1)
    res = {
        "metric": f"decoder-stack tok/s ({args.workload})", "value": B * args.steps / (ms * 1e-3), "unit": "tok/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 attention (tcgen05, f32 softmax) + e2m1 x e4m3 MoE (tcgen05)",
        "data": "synthetic (random-init attention / dense weights, random bf16 KV caches, seeded MXFP4 pools)",
        "config": workload_config(args.workload),
        "distinct_experts_per_step": step_U,
        "roofline": {"kernel": "whole decode step (attention weights, KV caches, dense MLP, routers, distinct experts)",
                     "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "peak_kind": f"{peak_kind} hbm_gbs", "traffic": None, "algorithmic_bytes_per_step": step_bytes},
        "clocks": clk,
        "e2e": {"value": B * e2e_steps / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": B * H * 2,
                "d2h_bytes_per_step": B * H * 2,
                "how": "eager DecoderStack call per step (host launches of every layer), pinned host x in, y out",
                "value_graph_replay": B * args.steps / (g_ms * 1e-3)},
        # per layer: rmsnorm, RoPE + cache, attention + split merge, add + RMSNorm, add, the q|k|v and o
        # projections with their segment sums; per MoE layer the block's five (route logits, select, gate/up,
        # down, combine); the dense layer's SwiGLU and its two projections
        "gpu_launches": (L * 10 + (L - 1) * 5 + 5) * args.steps,
        "cpu_baseline": None,
    }
    print(json.dumps(res))


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
    B, L = WORKLOADS[args.workload][0], args.layers
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
        c = cpu_baseline(f"decode{B}", args.cpu_budget)
        cpu = dict(c, value=c["value"] / L, sample=f"one layer's rate / {L} layers; {c['sample']}")
    if rank == 0:
        tok = B * args.steps * world
        # per layer: single GPU = route, gate/up, down, combine; peer exchange = router logits,
        # route+scatter, 2 barriers, unit builder, term split, gate/up, down, combine; plus one RMSNorm
        # between layers
        per_layer = (8 if world > 1 else 4) - (1 if fused else 0)
        out = {
            "metric": f"MoE-stack tok/s ({args.workload}, {L} layers)", "value": tok / (ms * 1e-3), "unit": "tok/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e2m1 x e4m3 (two-term activations) -> f32, tcgen05 block-scaled",
            "data": "synthetic (48 independently seeded MXFP4 layers, x ~ N(0,1) bf16, router W ~ N(0,0.02))",
            "config": dict(workload_config(args.workload, world), layers=L),
            "expert_bytes_per_gpu": L * (hi - lo) * EXPERT_BYTES,
            "mean_distinct_experts_per_layer": statistics.mean(U),
            "mean_distinct_experts_per_layer_this_gpu": statistics.mean(U_local),
            "graph": "the whole L-layer step is one CUDA graph",
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
                    "d2h_bytes_per_step": B * H * 2, "how": "graph replay of the stack, pinned x in, y out"},
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
    ap.add_argument("--no-nested", action="store_true", help="only the headline workload")
    ap.add_argument("--cpu-budget", type=float, default=4.0, help="seconds of timed CPU work per baseline variant")
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
    if args.workload.startswith("model"):
        return bench_model(args)
    import torch.distributed as dist
    ctx = Ctx(args)
    if args.workload.startswith("layer"):
        if ctx.world > 1:
            raise SystemExit("the decoder-layer workloads run on one GPU")
        print(json.dumps(measure_layer(args, ctx, args.workload, args.steps, args.warmup, args.cpu_budget)))
        return
    head = measure(args, ctx, args.workload, args.steps, args.warmup, args.cpu_budget, emulator=True)
    nested = {}
    if ctx.world == 1 and not args.no_nested and args.workload == "decode8" and args.pool_experts == E:
        for wl in NESTED:
            T = WORKLOADS[wl][0]
            k = args.steps if T <= 8 else max(10, min(args.steps, 40))
            nested[wl] = measure(args, ctx, wl, k, args.warmup, args.cpu_budget, emulator=False)
        for wl in LAYER_NESTED:
            T = WORKLOADS[wl][0]
            k = args.steps if T <= 8 else max(10, min(args.steps, 20))
            nested[wl] = measure_layer(args, ctx, wl, k, args.warmup, args.cpu_budget)
        head["configs"] = nested
    if ctx.rank == 0:
        print(json.dumps(head))
    if ctx.world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
