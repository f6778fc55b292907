"""The test kit's dense tensor peak probe (mimo_moe_tensor_peak): both MMA forms run to completion on
every SM and report a rate between the bf16 rate and twice the nominal FP4 rate of a B200, with the
FP4 form (kind::mxf4) at least as fast as the e2m1 x e4m3 form (kind::mxf8f6f4)."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_tensor_peak_probe(gpu):
    from mimo_moe import _lib
    L = _lib.testkit()
    status = torch.zeros(1, dtype=torch.int32, device=gpu)
    stream = torch.cuda.current_stream(gpu).cuda_stream
    rates = {}
    for kind in (0, 1):
        t = ctypes.c_float(0.0)
        for _ in range(2):
            assert L.mimo_moe_tensor_peak(kind, 2000, ctypes.byref(t), status.data_ptr(), stream) == 0
        rates[kind] = float(t.value)
    assert int(status.item()) == 0
    print(f"measured dense tensor peak: mxf8f6f4 {rates[0]:.0f} TFLOP/s, mxf4 {rates[1]:.0f} TFLOP/s")
    assert 1000.0 < rates[0] < 18000.0
    assert rates[1] >= 0.9 * rates[0]
    # arguments outside the probe's range are refused
    t = ctypes.c_float(0.0)
    assert L.mimo_moe_tensor_peak(2, 10, ctypes.byref(t), status.data_ptr(), stream) == 1
