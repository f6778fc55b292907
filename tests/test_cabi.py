"""C-ABI library checks that need no GPU: the block library and the test kit load, export every symbol
include/mimo_moe.h, include/mimo_moe_layer.h and include/mimo_moe_testkit.h declare, and their host-side argument checks reject
bad calls before touching the device."""
import ctypes
import re

import pytest
import torch

from conftest import ROOT


def declared_functions(header="mimo_moe.h"):
    hdr = (ROOT / "include" / header).read_text()
    hdr = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(mimo_moe_[a-z0-9_]+)\s*\(", hdr)))


def test_library_exports_every_declared_symbol():
    import mimo_moe
    L = mimo_moe.lib()
    names = declared_functions() + declared_functions("mimo_moe_layer.h")
    assert len(names) >= 21
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    from mimo_moe._lib import SIGNATURES, TESTKIT_SIGNATURES, testkit
    assert set(names) <= set(SIGNATURES), set(names) - set(SIGNATURES)
    kit = declared_functions("mimo_moe_testkit.h")
    K = testkit()
    assert kit and not [n for n in kit if not hasattr(K, n)]
    assert set(kit) == set(TESTKIT_SIGNATURES)
    assert not set(kit) & set(names)            # the block library does not carry the kit


def test_version_and_errors():
    import mimo_moe
    L = mimo_moe.lib()
    assert L.mimo_moe_version() == 1
    assert L.mimo_moe_strerror(0) == b"ok"
    assert b"range" in L.mimo_moe_strerror(2)


def test_workspace_sizes_are_host_only():
    import mimo_moe
    L = mimo_moe.lib()
    assert L.mimo_moe_experts_workspace_bytes(8, 64, 8, 4096, 2048) >= 8 * 4096 * 2 + 64 * 8 * (2048 * 2 + 4096 * 4)
    assert L.mimo_moe_prefill_workspace_bytes(2048, 8, 4096, 2048, 256) >= 2048 * 8 * (2048 * 2 + 4096 * 2)
    assert L.mimo_moe_block_workspace_bytes(1, 4096, 2048, 256, 8) > 0
    assert L.mimo_moe_dispatch_workspace_bytes(2048, 8, 256) == 8 * 256 * 4
    assert L.mimo_moe_experts_workspace_bytes(0, 1, 1, 4096, 2048) == 0


def test_bad_arguments_return_einval_without_a_device():
    import mimo_moe
    L = mimo_moe.lib()
    EINVAL = 1
    assert L.mimo_moe_router(None, None, None, 1, 4096, 256, 8, None, None, None, None) == EINVAL
    assert L.mimo_moe_topk(None, None, 1, 256, 8, None, None, None) == EINVAL
    assert L.mimo_moe_topk(1, None, 1, 300, 8, 1, 1, None) == EINVAL          # E > 256
    assert L.mimo_moe_topk(1, None, 1, 256, 9, 1, 1, None) == EINVAL          # topk > 8
    assert L.mimo_moe_group_routes(1, 1, 200, 8, 8, 256, 1, 1, 1, 1, 1, 1, None, None) == EINVAL  # M*k > 1024
    pools = mimo_moe._lib.Pools(1, 1, 1, 1, 1, 1, 256, 4096, 1000)           # I not a multiple of 2048
    assert L.mimo_moe_experts(1, ctypes.byref(pools), 1, 1, 1, 1, None, 8, 8, None, 8, 1, 0, 1, 1,
                              1 << 30, None, None) == EINVAL
    pools = mimo_moe._lib.Pools(1, 1, 1, 1, 1, 1, 256, 4096, 2048)
    assert L.mimo_moe_experts(1, ctypes.byref(pools), 1, 1, 1, 1, None, 8, 9, None, 8, 1, 0, 1, 1,
                              1 << 30, None, None) == EINVAL                   # R > 8
    assert L.mimo_moe_experts(1, ctypes.byref(pools), 1, 1, 1, 1, None, 8, 8, None, 8, 1, 0, 1, 1,
                              16, None, None) == EINVAL                        # workspace too small
    assert L.mimo_moe_prefill(1, ctypes.byref(pools), None, 100, 1, 1, 4, 8, 1, 1, 1 << 30, None,
                              None) == EINVAL                                  # E != S without slot_of
    K = mimo_moe._lib.testkit()
    assert K.mimo_moe_fill_synthetic_pool(None, None, None, None, None, None, 1, 4096, 2048, 0, 0, 0,
                                          None) == EINVAL
    assert L.mimo_moe_rmsnorm(None, None, 1, 4096, 1e-6, None, None) == EINVAL
    assert L.mimo_moe_rmsnorm(256, None, 1, 12, 1e-6, 256, None) == EINVAL       # H % 8
    assert L.mimo_moe_rmsnorm(264, None, 1, 4096, 1e-6, 256, None) == EINVAL     # x not 16-byte aligned
    assert L.mimo_moe_rmsnorm(256, None, 1, 4096, -1.0, 256, None) == EINVAL     # eps < 0
    assert L.mimo_moe_combine_pairs(None, None, None, 1, 8, 4096, None, None) == EINVAL
    assert L.mimo_moe_combine_pairs(256, 256, 256, 1, 9, 4096, 256, None) == EINVAL  # topk > 8
    assert L.mimo_moe_read_file_spans(None, None, 0, 1, 4096, 0, 1, None) == EINVAL     # no path
    assert L.mimo_moe_read_file_spans(b"/dev/null", None, 0, 0, 4096, 0, 1, None) == EINVAL  # 0 threads
    assert L.mimo_moe_read_file_spans(b"/dev/null", None, 0, 1, 5000, 0, 1, None) == EINVAL  # chunk % 4096
    assert L.mimo_moe_read_file_spans(b"/dev/null", None, 0, 1, 4096, 0, 1, None) == 0       # nothing to read


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: host tensors are rejected."""
    import mimo_moe
    x = torch.zeros(1, 4096, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        mimo_moe.router(x, torch.zeros(256, 4096, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        mimo_moe.group_routes(torch.zeros(1, 8, dtype=torch.int32), torch.zeros(1, 8))
