"""Failure detection on the GPU without a GPU fault: a bounded wait that runs
out (a barrier nothing arrives on) reports MB_ERR_TIMEOUT through the device
status word, and the context keeps working afterwards."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives():
    import torch
    from metalbench_b200 import _lib, ops
    ops.init(0)
    L = _lib.lib()
    _lib.call("mb_clear_device_status")
    rc = L.mb_selftest_bounded_wait(20000, None)  # 20 ms limit
    assert rc == -5 and "timed out" in _lib.last_error()
    v = C.c_uint32(0)
    _lib.call("mb_device_status", C.byref(v))
    assert v.value & 0x100
    _lib.call("mb_clear_device_status")
    _lib.call("mb_device_status", C.byref(v))
    assert v.value == 0
    a = torch.randn(256, 192, device="cuda")  # the context is still usable
    assert torch.equal(ops.transpose_2d(a), a.t().contiguous())


def test_run_reports_bad_arguments_without_launch():
    from metalbench_b200 import _lib
    L = _lib.lib()
    rc = L.mb_gemm_bf16(None, None, None, 64, 12, 64, 0, None)  # N % 8 != 0
    assert rc == -1 and "multiple of 8" in _lib.last_error()
    rc = L.mb_conv2d_nhwc_bf16(None, None, None, 1, 8, 8, 64, 64, 3, 3, 2, 1, None)
    assert rc == -1 and "stride" in _lib.last_error()
