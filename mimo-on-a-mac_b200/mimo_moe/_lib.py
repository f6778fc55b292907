"""ctypes bindings of libmimo_moe.so (the C ABI in include/mimo_moe.h and include/mimo_moe_layer.h) and of the test and benchmark
kit beside it, libmimo_moe_testkit.so (include/mimo_moe_testkit.h: synthetic pools, tensor-peak probe).

There is no CPU fallback: if the library is missing or cannot be loaded, every op raises."""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int32, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(os.environ.get("MIMO_MOE_LIBRARY") or Path(__file__).resolve().with_name("libmimo_moe.so"))
TESTKIT_PATH = Path(__file__).resolve().with_name("libmimo_moe_testkit.so")

MIMO_OK, MIMO_EINVAL, MIMO_ERANGE, MIMO_ETIMEOUT, MIMO_ECUDA, MIMO_EIO = 0, 1, 2, 3, 4, 5


class Pools(ctypes.Structure):
    """struct mimo_moe_pools."""
    _fields_ = [("gate_w", c_void_p), ("gate_s", c_void_p), ("up_w", c_void_p), ("up_s", c_void_p),
                ("down_w", c_void_p), ("down_s", c_void_p), ("num_slots", c_int32),
                ("hidden", c_int32), ("inter", c_int32)]


# name -> (restype, argtypes)
SIGNATURES = {
    "mimo_moe_version": (c_int32, []),
    "mimo_moe_strerror": (ctypes.c_char_p, [c_int32]),
    "mimo_moe_last_cuda_error": (c_int32, []),
    "mimo_moe_router": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                  c_void_p, c_void_p, c_void_p, c_void_p]),
    "mimo_moe_topk": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p,
                                c_void_p]),
    "mimo_moe_group_routes": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_void_p]),
    "mimo_moe_dispatch_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "mimo_moe_dispatch": (c_int32, [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_size_t, c_void_p, c_void_p]),
    "mimo_moe_ep_plan_workspace_bytes": (c_size_t, [c_int32, c_int32]),
    "mimo_moe_ep_plan": (c_int32, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "mimo_moe_gather_rows": (c_int32, [c_void_p, c_int64, c_int32, c_void_p, c_int64, c_void_p, c_void_p,
                                       c_void_p]),
    "mimo_moe_ep_recv_index": (c_int32, [c_void_p, c_void_p, c_int32, c_int64, c_void_p, c_void_p, c_void_p,
                                         c_void_p]),
    "mimo_moe_prefill_routes": (c_int32, [c_void_p, c_int32, POINTER(Pools), c_void_p, c_int32, c_void_p,
                                          c_void_p, c_int32, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "mimo_moe_experts_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "mimo_moe_experts": (c_int32, [c_void_p, POINTER(Pools), c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_void_p, c_int32, c_int32, c_void_p, c_int32, c_int32, c_int32,
                                   c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "mimo_moe_prefill_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "mimo_moe_experts_routes_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "mimo_moe_experts_routes": (c_int32, [c_void_p, c_int32, c_int32, POINTER(Pools), c_int32, c_void_p,
                                          c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_int32,
                                          c_void_p, c_size_t, c_void_p, c_void_p]),
    "mimo_moe_slot_cache_create": (c_void_p, [c_int32, c_int32]),
    "mimo_moe_slot_cache_destroy": (None, [c_void_p]),
    "mimo_moe_slot_cache_preload": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p]),
    "mimo_moe_slot_cache_resolve": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p,
                                              c_void_p]),
    "mimo_moe_slot_cache_decay": (c_int32, [c_void_p]),
    "mimo_moe_slot_cache_state": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "mimo_moe_peer_alloc": (c_int32, [c_size_t, c_void_p, c_void_p]),
    "mimo_moe_peer_open": (c_int32, [c_void_p, c_void_p]),
    "mimo_moe_peer_close": (c_int32, [c_void_p]),
    "mimo_moe_peer_free": (c_int32, [c_void_p]),
    "mimo_moe_peer_barrier": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int32, c_void_p,
                                        c_void_p]),
    "mimo_moe_route_scatter": (c_int32, [c_void_p, c_int32, c_int32, c_void_p, c_void_p, c_int32, c_int32,
                                         c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p]),
    "mimo_moe_combine": (c_int32, [c_void_p, ctypes.c_int64, c_void_p, c_int32, c_int32, c_int32, c_void_p,
                                   c_void_p, c_void_p]),
    "mimo_moe_read_file_spans": (c_int32, [ctypes.c_char_p, c_void_p, c_int32, c_int32, ctypes.c_int64, c_int32,
                                           c_int32, c_void_p]),
    "mimo_moe_rmsnorm": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_float, c_void_p, c_void_p]),
    "mimo_moe_combine_pairs": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p,
                                         c_void_p]),
    "mimo_moe_prefill": (c_int32, [c_void_p, POINTER(Pools), c_void_p, c_int32, c_void_p, c_void_p,
                                   c_int32, c_int32, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "mimo_moe_block_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "mimo_moe_block": (c_int32, [c_void_p, c_void_p, c_void_p, POINTER(Pools), c_int32, c_int32,
                                 c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p, c_void_p]),
    "mimo_moe_experts_static_scratch_bytes": (c_size_t, []),
    "mimo_moe_experts_static": (c_int32, [c_void_p, POINTER(Pools), c_void_p, c_void_p, c_void_p,
                                          c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int32,
                                          c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    "mimo_moe_layer_rope_store": (c_int32, [c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_float,
                                            c_float, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p]),
    "mimo_moe_layer_attention_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32]),
    "mimo_moe_layer_attention": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                           c_int32, c_int32, c_float, c_int32, c_int32, c_int32, c_int32, c_void_p,
                                           c_void_p, c_size_t, c_void_p, c_void_p]),
    "mimo_moe_layer_linear_workspace_bytes": (c_size_t, [c_int32, c_int32, c_int32]),
    "mimo_moe_layer_linear": (c_int32, [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p, c_size_t,
                                        c_void_p, c_void_p]),
    "mimo_moe_layer_add_rmsnorm": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_float, c_void_p,
                                             c_void_p, c_void_p]),
    "mimo_moe_layer_swiglu": (c_int32, [c_void_p, c_int32, c_int32, c_void_p, c_void_p]),
    "mimo_moe_layer_add": (c_int32, [c_void_p, c_void_p, c_int64, c_void_p, c_void_p]),
    "mimo_moe_profile_enable": (c_int32, [c_int32]),
    "mimo_moe_profile_read": (c_int32, [c_void_p, c_void_p]),
}
TESTKIT_SIGNATURES = {
    "mimo_moe_tensor_peak": (c_int32, [c_int32, c_int32, c_void_p, c_void_p, c_void_p]),
    "mimo_moe_fill_synthetic_pool": (c_int32, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                               c_void_p, c_int32, c_int32, c_int32, c_uint64, c_int32,
                                               c_int32, c_void_p]),
}

_lib = None
_testkit = None


def _load(path: Path, signatures: dict) -> ctypes.CDLL:
    if not path.exists():
        raise RuntimeError(f"mimo_moe: CUDA library not built ({path}); run "
                           "`python mimo-on-a-mac_b200/mimo_moe/build.py` or __graft_entry__.build()")
    L = ctypes.CDLL(str(path))
    for name, (res, args) in signatures.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


def lib() -> ctypes.CDLL:
    """Load the CUDA library (raises RuntimeError when it is absent: there is no fallback)."""
    global _lib
    if _lib is None:
        _lib = _load(LIB_PATH, SIGNATURES)
    return _lib


def testkit() -> ctypes.CDLL:
    """Load the test and benchmark kit (synthetic pools, tensor-peak probe)."""
    global _testkit
    if _testkit is None:
        lib()  # the block library first: the kit shares its error codes
        _testkit = _load(TESTKIT_PATH, TESTKIT_SIGNATURES)
    return _testkit


class MimoError(RuntimeError):
    def __init__(self, code: int, where: str):
        L = lib()
        msg = L.mimo_moe_strerror(code).decode()
        if code == MIMO_ECUDA:
            msg += f" (cudaError {L.mimo_moe_last_cuda_error()})"
        super().__init__(f"{where}: {msg}")
        self.code = code


def check(code: int, where: str) -> None:
    if code == MIMO_OK:
        return
    if code == MIMO_EINVAL:
        raise ValueError(f"{where}: {lib().mimo_moe_strerror(code).decode()}")
    raise MimoError(code, where)
