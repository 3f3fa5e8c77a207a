"""GPU parity of the implicit-GEMM conv2d against the oracle
(oracle.ops.conv2d_nhwc, mlx/kernels/common/conv2d.py:7-12) on bf16 inputs.
Gate: every element within |a-b| <= 2e-2*|b| + 2e-2*rms(b) (bf16 output)."""
import numpy as np
import pytest

import oracle.ops as O

pytestmark = pytest.mark.gpu


def _bf16(torch, x):
    return torch.from_numpy(O.f32_to_bf16(x).view(np.int16)).cuda().view(torch.bfloat16)


@pytest.mark.parametrize("xs,ws,pad", [
    ((32, 56, 56, 64), (64, 3, 3, 64), 1),     # BASELINE config
    ((8, 64, 64, 64), (128, 3, 3, 64), 0),     # reference registry shape
    ((1, 5, 7, 64), (16, 3, 3, 64), 1),        # tiny, ragged
    ((2, 20, 130, 128), (256, 3, 3, 128), 1),  # W2 > 64 tiles, 2 channel chunks
    ((2, 9, 9, 64), (48, 1, 1, 64), 0),        # 1x1, Cout not a multiple of 32
    ((1, 12, 11, 64), (32, 5, 5, 64), 2),      # 5x5
    ((0, 8, 8, 64), (64, 3, 3, 64), 1),        # empty batch
    ((3, 17, 23, 64), (32, 3, 3, 64), 1),      # resident path, 25-slot position rows
    ((2, 30, 62, 64), (64, 3, 3, 64), 1),      # resident path, 64-slot rows (the widest)
    ((2, 4, 1, 64), (64, 3, 1, 64), 0),        # resident path, 1-slot rows, 3x1 filter
])
def test_conv2d_bf16(xs, ws, pad):
    import torch
    from metalbench_b200 import ops
    rng = np.random.default_rng(2)
    x = O.round_bf16(rng.standard_normal(xs).astype(np.float32))
    w = O.round_bf16((rng.standard_normal(ws) * np.sqrt(2.0 / (ws[1] * ws[2] * ws[3]))).astype(np.float32))
    y = ops.conv2d_nhwc(_bf16(torch, x), _bf16(torch, w), padding=pad)
    got = O.bf16_to_f32(y.view(torch.int16).cpu().numpy().view(np.uint16))
    ref = O.conv2d_nhwc(x, w, padding=pad)
    assert got.shape == ref.shape
    if ref.size == 0:
        return
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    r = O.allclose_report(got, ref, rtol=2e-2, atol=2e-2 * rms)
    assert r["all"], r


def test_conv2d_rejects_stride2():
    import torch
    from metalbench_b200 import ops, _lib
    x = torch.zeros((1, 8, 8, 64), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((64, 3, 3, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.MbError):
        ops.conv2d_nhwc(x, w, stride=2, padding=1)


@pytest.mark.parametrize("path", ["resident", "tiled"])
@pytest.mark.parametrize("xs,pad", [((32, 56, 56, 64), 1), ((3, 13, 40, 64), 1),
                                    ((2, 10, 64, 64), 0)])
def test_conv2d_both_paths(xs, pad, path, monkeypatch):
    """The resident-weight path (weights loaded once per CTA, one TMA box per
    filter column) and the per-tap tiled path agree with the oracle."""
    import torch
    from metalbench_b200 import ops
    if path == "tiled":
        monkeypatch.setenv("MB_CONV_NO_RESIDENT", "1")
    rng = np.random.default_rng(12)
    ws = (64, 3, 3, xs[3])
    x = O.round_bf16(rng.standard_normal(xs).astype(np.float32))
    w = O.round_bf16((rng.standard_normal(ws) * np.sqrt(2.0 / 576)).astype(np.float32))
    y = ops.conv2d_nhwc(_bf16(torch, x), _bf16(torch, w), padding=pad)
    got = O.bf16_to_f32(y.view(torch.int16).cpu().numpy().view(np.uint16))
    ref = O.conv2d_nhwc(x, w, padding=pad)
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    r = O.allclose_report(got, ref, rtol=2e-2, atol=2e-2 * rms)
    assert r["all"], r
