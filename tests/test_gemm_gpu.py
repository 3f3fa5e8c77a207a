"""GPU parity of the tcgen05 GEMMs.

* ``sqr_mm`` (fp32, 3xTF32) against the float64 oracle (oracle.ops.sqr_mm,
  mlx/kernels/common/sqr_mm.py:10-11): relative error <= 1e-4.
* ``gemm_bf16`` against the oracle on bf16-rounded inputs: every element within
  |a-b| <= 2e-2*|b| + 2e-2*rms(b) (north-star bf16 tolerance), and >= 99 %.
"""
import numpy as np
import pytest

import oracle.ops as O

pytestmark = pytest.mark.gpu


def _bf16_tensor(torch, x):
    return torch.from_numpy(O.f32_to_bf16(x).view(np.int16)).cuda().view(torch.bfloat16)


def _to_np(t):
    import torch
    if t.dtype == torch.bfloat16:
        return O.bf16_to_f32(t.view(torch.int16).cpu().numpy().view(np.uint16))
    return t.cpu().numpy()


def _gate(got, ref, rtol, atol_rel_rms):
    atol = atol_rel_rms * float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)) or 1.0)
    r = O.allclose_report(got, ref, rtol=rtol, atol=atol)
    return r


@pytest.mark.parametrize("M,N,K", [(2048, 2048, 2048), (256, 256, 128), (130, 72, 36),
                                   (1, 4, 4), (384, 640, 1000), (1024, 2048, 4096)])
def test_sqr_mm_f32_3xtf32(M, N, K):
    import torch
    from metalbench_b200 import ops
    rng = np.random.default_rng(0)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    C = ops.sqr_mm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    got = C.cpu().numpy()
    ref = O.sqr_mm(A, B, acc=np.float64)
    rel = np.abs(got - ref).max() / np.abs(ref).max()
    assert rel <= 1e-4, rel
    r = _gate(got, ref, rtol=1e-4, atol_rel_rms=1e-4)
    assert r["frac_within_tol"] >= 0.99, r


@pytest.mark.parametrize("b_layout", ["kn", "nk"])
@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (512, 768, 640), (200, 136, 72),
                                   (1, 8, 8), (4096, 4096, 4096), (128, 6144, 4096)])
def test_gemm_bf16(M, N, K, b_layout):
    import torch
    from metalbench_b200 import ops
    rng = np.random.default_rng(4)
    A = O.round_bf16(rng.standard_normal((M, K)).astype(np.float32))
    B = O.round_bf16(rng.standard_normal((K, N)).astype(np.float32))
    Bt = B if b_layout == "kn" else np.ascontiguousarray(B.T)
    C = ops.gemm_bf16(_bf16_tensor(torch, A), _bf16_tensor(torch, Bt), b_layout=b_layout)
    got = _to_np(C)
    if M * N * K <= 2 ** 31:
        ref = O.sqr_mm(A, B, acc=np.float64)
    else:  # torch fp32 reference of the same op for the large case (TF32 off)
        torch.backends.cuda.matmul.allow_tf32 = False
        ref = (torch.from_numpy(A).cuda() @ torch.from_numpy(B).cuda()).cpu().numpy()
    r = _gate(got, ref, rtol=2e-2, atol_rel_rms=2e-2)
    assert r["all"], r


def test_gemm_bf16_layouts_agree_bitwise():
    """The MN-major and K-major B paths feed the same products to the same
    accumulator order, so their outputs are identical."""
    import torch
    from metalbench_b200 import ops
    rng = np.random.default_rng(5)
    A = rng.standard_normal((512, 1024)).astype(np.float32)
    B = rng.standard_normal((1024, 512)).astype(np.float32)
    a = _bf16_tensor(torch, A)
    c1 = ops.gemm_bf16(a, _bf16_tensor(torch, B), b_layout="kn")
    c2 = ops.gemm_bf16(a, _bf16_tensor(torch, np.ascontiguousarray(B.T)), b_layout="nk")
    assert torch.equal(c1.view(torch.int16), c2.view(torch.int16))


def test_gemm_device_status_clean():
    from metalbench_b200 import _lib
    import ctypes as C
    v = C.c_uint32(7)
    _lib.call("mb_device_status", C.byref(v))
    assert v.value == 0


@pytest.mark.parametrize("M,N,K", [(1024, 2048, 4096), (512, 512, 16384)])
def test_sqr_mm_f32_elementwise_gate_deep_k(M, N, K):
    """Every element within the registry's fp32 gate (|a-b| <= 1e-3 + 1e-4|b|)
    of the float64 product, also at deep K: the tensor-core partial sums are
    restarted every 128 of K and added in fp32 registers."""
    import torch
    from metalbench_b200 import ops
    rng = np.random.default_rng(6)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    got = ops.sqr_mm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()).cpu().numpy()
    ref = A.astype(np.float64) @ B.astype(np.float64)
    r = O.allclose_report(got, ref, rtol=1e-4, atol=1e-3)
    assert r["all"], r


@pytest.mark.parametrize("batch,M,N,K", [(128, 128, 512, 256), (3, 256, 200, 64), (5, 100, 72, 36),
                                         (1, 128, 128, 128)])
def test_batch_mm_f32(batch, M, N, K):
    """batch_mm (one launch over all batches when M % 128 == 0, else batch by
    batch) against the float64 product, fp32 gate on every element."""
    import torch
    from metalbench_b200 import ops
    rng = np.random.default_rng(7)
    A = rng.standard_normal((batch, M, K)).astype(np.float32)
    B = rng.standard_normal((batch, K, N)).astype(np.float32)
    got = ops.batch_mm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()).cpu().numpy()
    ref = np.matmul(A.astype(np.float64), B.astype(np.float64))
    r = O.allclose_report(got, ref, rtol=1e-4, atol=1e-3)
    assert r["all"], r
