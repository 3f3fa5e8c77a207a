"""GPU parity of the transpose kernels against the oracle (bit-exact).

Registry reference: mlx/kernels/common/registry.py:165-179 (rtol = atol = 0).
"""
import ctypes as C

import numpy as np
import pytest

import oracle.ops as O

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


@pytest.mark.parametrize("rows,cols", [(8192, 8192), (1024, 2048), (48, 80), (33, 17), (1, 1),
                                       (65, 130), (64, 64), (128, 4), (4, 128), (3, 1000),
                                       (0, 5), (130, 66)])
def test_transpose_2d_f32_bit_exact(rows, cols):
    torch = _torch()
    from metalbench_b200 import ops
    rng = np.random.default_rng(1)
    a = rng.uniform(-1, 1, (rows, cols)).astype(np.float32)
    out = ops.transpose_2d(torch.from_numpy(a).cuda())
    torch.cuda.synchronize()
    assert out.cpu().numpy().tobytes() == O.transpose_2d(a).tobytes()


@pytest.mark.parametrize("shape", [(64, 1024, 1024), (3, 100, 72), (2, 9, 7), (1, 64, 64),
                                   (5, 136, 264), (2, 8, 16)])
def test_transpose_batched_bf16_bit_exact(shape):
    torch = _torch()
    from metalbench_b200 import ops
    rng = np.random.default_rng(1)
    bits = O.f32_to_bf16(rng.uniform(-1, 1, shape).astype(np.float32))
    a = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    out = ops.transpose_batched(a)
    torch.cuda.synchronize()
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    assert got.tobytes() == O.transpose_2d(bits).tobytes()


def test_transpose_batched_f32_bit_exact():
    torch = _torch()
    from metalbench_b200 import ops
    a = np.random.default_rng(3).standard_normal((4, 200, 96)).astype(np.float32)
    out = ops.transpose_batched(torch.from_numpy(a).cuda())
    assert out.cpu().numpy().tobytes() == O.transpose_2d(a).tobytes()


def test_transpose_special_values_preserved():
    torch = _torch()
    from metalbench_b200 import ops
    a = np.array([[np.nan, -0.0, np.inf, -np.inf], [1e-45, 3.4e38, 0.0, -1.0]] * 32, np.float32)
    out = ops.transpose_2d(torch.from_numpy(a).cuda()).cpu().numpy()
    assert out.tobytes() == np.ascontiguousarray(a.T).tobytes()


def test_mb_run_manifest_path_host_buffers():
    """The reference-facing manifest entry point with host buffers."""
    from metalbench_b200 import _lib
    L = _lib.lib()
    _lib.call("mb_init", 0, 0, 1, None, 0)
    rows, cols = 1024, 2048
    a = np.random.default_rng(1).uniform(-1, 1, (rows, cols)).astype(np.float32)
    out = np.empty((cols, rows), np.float32)
    bufs = (_lib.MbBuf * 2)(
        _lib.MbBuf(0, _lib.ROLE_INPUT, _lib.DTYPE["f32"], 0, a.ctypes.data, a.nbytes),
        _lib.MbBuf(1, _lib.ROLE_OUTPUT, _lib.DTYPE["f32"], 0, out.ctypes.data, out.nbytes))
    sc = (_lib.MbScalar * 2)()
    sc[0].binding, sc[0].dtype, sc[0].v.u = 2, _lib.DTYPE["u32"], rows
    sc[1].binding, sc[1].dtype, sc[1].v.u = 3, _lib.DTYPE["u32"], cols
    t = _lib.MbTiming()
    _lib.check("mb_run", L.mb_run(b"transpose_2d", bufs, 2, sc, 2, b'{"flush_l2": true}', 2, 5,
                                  C.byref(t)))
    assert out.tobytes() == O.transpose_2d(a).tobytes()
    assert t.iters == 5 and 0 < t.min_ms <= t.median_ms


def test_mb_run_rejects_wrong_sizes():
    from metalbench_b200 import _lib
    L = _lib.lib()
    _lib.call("mb_init", 0, 0, 1, None, 0)
    a = np.zeros((4, 4), np.float32)
    out = np.zeros((4, 4), np.float32)
    bufs = (_lib.MbBuf * 2)(
        _lib.MbBuf(0, _lib.ROLE_INPUT, 0, 0, a.ctypes.data, a.nbytes),
        _lib.MbBuf(1, _lib.ROLE_OUTPUT, 0, 0, out.ctypes.data, out.nbytes))
    sc = (_lib.MbScalar * 2)()
    sc[0].binding, sc[0].dtype, sc[0].v.u = 2, 3, 8
    sc[1].binding, sc[1].dtype, sc[1].v.u = 3, 3, 8
    rc = L.mb_run(b"transpose_2d", bufs, 2, sc, 2, None, 0, 1, None)
    assert rc == -1 and "size" in _lib.last_error()
    rc = L.mb_run(b"no_such_kernel", bufs, 2, sc, 2, None, 0, 1, None)
    assert rc == -2
