"""Multi-GPU expert-parallel check, one process per GPU (launched by tests/test_ep_multi_gpu.py):

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 tests/ep_worker.py

Rank r holds experts [r*256/N, (r+1)*256/N) of a seeded synthetic layer, routes its own T tokens and
runs the expert-parallel block (mimo_moe/ep.py, NCCL).  Each rank then runs the single-GPU block on
the same tokens with the whole layer resident and the outputs must be identical bit for bit, for
T = 1 (stock-path rounding), 8 (decode) and 12 (prefill rounding) through the NCCL all-gather block,
T = 1 and 8 through the peer-memory block (eager and graphed), and T = 64 and 600 through the
all-to-all prefill block, and a 3-layer decode stack over the peer exchange at T = 1 and 8 against
the single-GPU stack.  Prints one JSON line per rank."""
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "mimo-on-a-mac_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import mimo_moe  # noqa: E402
from mimo_moe.ep import (ExpertParallelMoE, ExpertParallelPrefill, GraphedStep,  # noqa: E402
                         PeerExpertParallelMoE, expert_range)
from oracle import synth  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    ok = True
    res = {"rank": rank, "world": world}
    try:
        lo, hi = expert_range(rank, world)
        shard = mimo_moe.ExpertPools.synthetic(hi - lo, seed=0, layer=3, first_expert=lo, device=dev)
        full = mimo_moe.ExpertPools.synthetic(256, seed=0, layer=3, device=dev)
        W = synth.router_weight().to(dev)
        bias = torch.zeros(256, device=dev)
        blk = ExpertParallelMoE(shard, W, bias)
        for T in (1, 8, 12):
            x = synth.hidden(T, seed=500 + 17 * rank + T).to(dev)
            y_ep = blk(x)
            y_1 = mimo_moe.moe_block(x, W, bias, full)
            torch.cuda.synchronize()
            same = bool(torch.equal(y_ep.view(torch.int16), y_1.view(torch.int16)))
            res[f"T{T}_bit_identical"] = same
            ok &= same
        # the peer-memory exchange (decode sizes), eager and as a replayed CUDA graph
        for T in (1, 8):
            peer = PeerExpertParallelMoE(shard, W, bias, T)
            g = GraphedStep(peer, T, 4096, dev)
            for rep in range(3):
                x = synth.hidden(T, seed=900 + 31 * rank + 7 * rep + T).to(dev)
                y_1 = mimo_moe.moe_block(x, W, bias, full)
                y_p = peer(x).clone()
                y_g = g(x).clone()
                torch.cuda.synchronize()
                same = bool(torch.equal(y_p.view(torch.int16), y_1.view(torch.int16)) and
                            torch.equal(y_g.view(torch.int16), y_1.view(torch.int16)))
                res[f"peer_T{T}_rep{rep}_bit_identical"] = same
                ok &= same
            res[f"peer_T{T}_status"] = int(peer.status.item())
            ok &= res[f"peer_T{T}_status"] == 0
            del g
            peer.close()
        # a 3-layer decode stack (RMSNorm between layers): one peer exchange serves every layer
        from mimo_moe.stack import MoEStack
        lay_full, lay_shard = [], []
        for l in range(3):
            Wl = synth.router_weight(seed=1 + 1000 * l).to(dev)
            lay_full.append((Wl, None, mimo_moe.ExpertPools.synthetic(256, seed=0, layer=10 + l, device=dev)))
            lay_shard.append((Wl, None, mimo_moe.ExpertPools.synthetic(hi - lo, seed=0, layer=10 + l,
                                                                        first_expert=lo, device=dev)))
        single = MoEStack(lay_full)
        for T in (1, 8):
            ex = PeerExpertParallelMoE(lay_shard[0][2], lay_shard[0][0], None, T)
            st = MoEStack(lay_shard, layer_fn=lambda x, l, ex=ex: ex.layer(x, lay_shard[l][2], lay_shard[l][0], None))
            g = GraphedStep(st, T, 4096, dev)
            for rep in range(2):
                x = synth.hidden(T, seed=1300 + 31 * rank + 7 * rep + T).to(dev)
                y_1 = single(x).clone()
                y_g = g(x).clone()
                torch.cuda.synchronize()
                same = bool(torch.equal(y_g.view(torch.int16), y_1.view(torch.int16)))
                res[f"stack3_T{T}_rep{rep}_bit_identical"] = same
                ok &= same
            ok &= int(ex.status.item()) == 0
            del g
            ex.close()
        del lay_full, lay_shard, single
        # prefill sizes: each route travels to its expert's rank and back (NCCL all-to-all)
        pre = ExpertParallelPrefill(shard, W, bias)
        for T in (64, 600):
            x = synth.hidden(T, seed=700 + 13 * rank + T).to(dev)
            y_ep = pre(x)
            y_1 = mimo_moe.moe_block(x, W, bias, full)
            torch.cuda.synchronize()
            same = bool(torch.equal(y_ep.view(torch.int16), y_1.view(torch.int16)))
            res[f"prefill_T{T}_bit_identical"] = same
            ok &= same
    finally:
        dist.barrier()
        dist.destroy_process_group()
    print(json.dumps(res), flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
