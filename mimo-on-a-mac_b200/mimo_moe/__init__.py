"""B200-native (sm_100a) MiMo MoE block: router -> dispatch -> MXFP4 expert products -> combine.

Drop-in for the expert path of cialanjcampbell-coder/mimo-on-a-mac's engine/mimo_stream
(Router, group_routes, moe_experts, the gather_qmm pair path).  All compute runs in hand-written CUDA
(libmimo_moe.so, C ABI in include/mimo_moe.h); there is no CPU fallback."""
from ._lib import LIB_PATH, MimoError, lib
from .ops import (ExpertPools, Groups, MoEBlock, MoEConfig, Router, combine, combine_pairs, dispatch, group_routes,
                  moe_block, moe_experts, moe_experts_routes, moe_prefill, read_status, rmsnorm, router, topk)
from .loader import ExpertFile, load_expert_pools, load_router, save_expert_file
from .residency import ExpertCache, SlotCache
from .stack import MoEStack

__all__ = ["LIB_PATH", "MimoError", "lib", "ExpertCache", "ExpertFile", "ExpertPools", "Groups", "MoEBlock", "MoEConfig",
           "MoEStack", "Router", "SlotCache",
           "combine", "combine_pairs", "dispatch", "group_routes", "moe_block", "moe_experts", "moe_experts_routes",
           "load_expert_pools", "load_router", "moe_prefill", "read_status", "rmsnorm", "router",
           "save_expert_file", "topk"]
