"""mb_sqr_mm_f32_noalloc: sqr_mm for callers that cannot allocate device memory.

Such callers (a plugin inside a host process that owns every allocation, or
code running under a memory cap where cudaMalloc may fail or synchronise)
still need scratch space for the tf32 hi/lo splits. The entry point takes it
from a fixed 64 MiB array inside libmb200.so. This test calls it through the
C ABI and checks it against the caller-workspace entry point (mb_sqr_mm_f32,
via ops.sqr_mm) on two calls in a row, with the same tolerance as the other
sqr_mm tests (relative error <= 1e-4). It lives in its own file, collected
last, and works both alone in a fresh process and after the other tests.
"""
import numpy as np
import pytest

import oracle.ops as O

pytestmark = pytest.mark.gpu


def _noalloc(a, b, out):
    import torch
    from metalbench_b200 import _lib
    M, K = a.shape
    N = b.shape[1]
    rc = _lib.lib().mb_sqr_mm_f32_noalloc(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K,
                                          torch.cuda.current_stream().cuda_stream)
    _lib.check("mb_sqr_mm_f32_noalloc", rc)
    return out


def test_noalloc_matches_workspace_entry_point_twice():
    import torch
    from metalbench_b200 import ops
    rng = np.random.default_rng(11)
    for (M, N, K) in [(2048, 2048, 2048), (384, 640, 1000)]:  # two calls in a row
        A = rng.standard_normal((M, K)).astype(np.float32)
        B = rng.standard_normal((K, N)).astype(np.float32)
        a = torch.from_numpy(A).cuda()
        b = torch.from_numpy(B).cuda()
        ref = ops.sqr_mm(a, b).cpu().numpy()
        out = torch.full((M, N), float("nan"), device="cuda")
        got = _noalloc(a, b, out).cpu().numpy()
        rel = np.abs(got - ref).max() / np.abs(ref).max()
        assert rel <= 1e-4, rel
        truth = O.sqr_mm(A, B, acc=np.float64)
        assert np.abs(got - truth).max() / np.abs(truth).max() <= 1e-4
        # a clean call leaves no bounded-wait timeout on the device
        import ctypes
        from metalbench_b200 import _lib
        st = ctypes.c_uint32(1)
        assert _lib.lib().mb_device_status(ctypes.byref(st)) == 0 and st.value == 0


def test_noalloc_rejects_shapes_beyond_the_fixed_array():
    import torch
    from metalbench_b200 import _lib
    L = _lib.lib()
    limit = L.mb_sqr_mm_f32_noalloc_max_workspace_bytes()
    assert limit == 64 << 20
    M = N = K = 4096  # needs 256 MiB of scratch
    assert L.mb_sqr_mm_f32_workspace_bytes(M, N, K) > limit
    a = torch.empty((16,), device="cuda")  # pointers are never dereferenced
    rc = L.mb_sqr_mm_f32_noalloc(a.data_ptr(), a.data_ptr(), a.data_ptr(), M, N, K, None)
    assert rc == -1 and "fixed" in _lib.last_error()

