"""fp32 paths for the reference's own fp32 registry entries: conv2d_f32
(mlx/kernels/common/registry.py:469-477) and llama_decoder_layer_f32
(mlx/kernels/full/registry.py:87-104, head_dim 32), against the golden
fixtures the reference hooks produced and against the float64 oracle.
Gate: the reference's own, every element within atol + rtol*|b|
(mlx/scripts/harness.py:26-33), with the registry tolerances (1e-3 for
conv2d, 1e-2 for the decoder)."""
import numpy as np
import pytest

import oracle.ops as O
from _f32check import all_within as _all_within, check_against_fp32_golden

pytestmark = pytest.mark.gpu
REPO = __import__("pathlib").Path(__file__).resolve().parents[1]


def _t(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def test_conv2d_f32_golden():
    import torch
    from metalbench_b200 import ops
    g = np.load(REPO / "tests" / "golden" / "conv2d.npz")
    y = ops.conv2d_nhwc(_t(torch, g["in0"]), _t(torch, g["in1"]), padding=0)
    _all_within(y.cpu().numpy(), g["out"], 1e-3)


@pytest.mark.parametrize("N,H,W,C,Co,K,stride,pad", [
    (8, 64, 64, 64, 128, 3, 1, 0),    # the reference registry shape
    (3, 17, 23, 12, 40, 3, 2, 1),     # ragged, stride 2, padded
    (2, 9, 9, 8, 8, 5, 1, 2),         # 5x5, Cout < one tile
    (1, 7, 5, 4, 3, 1, 1, 0),         # 1x1, tiny
])
def test_conv2d_f32_matches_oracle(N, H, W, C, Co, K, stride, pad):
    import torch
    from metalbench_b200 import ops
    rng = np.random.default_rng(N * 100 + H)
    x = rng.standard_normal((N, H, W, C), dtype=np.float32)
    w = rng.standard_normal((Co, K, K, C), dtype=np.float32)
    y = ops.conv2d_nhwc(_t(torch, x), _t(torch, w), stride=stride, padding=pad)
    want = O.conv2d_nhwc(x, w, stride=stride, padding=pad, acc=np.float64)
    _all_within(y.cpu().numpy(), want, 1e-3)


def test_llama_decoder_f32_golden():
    """The reference registry's own shape: S 64, D 128, H 4 / H_kv 2 (head_dim 32)."""
    import torch
    from metalbench_b200 import ops
    g = np.load(REPO / "tests" / "golden" / "llama_decoder_layer.npz")
    ins = [_t(torch, g[f"in{i}"]) for i in range(5)]
    y = ops.llama_decoder_f32(*ins, n_heads=4, n_kv_heads=2, base=10000.0, eps=1e-5)
    exact = O.decoder_layer(g["in0"], *[g[f"in{i}"] for i in range(1, 5)], H=4, H_kv=2,
                            base=10000.0, acc=np.float64)
    check_against_fp32_golden(y.cpu().numpy(), g["out"], exact, 1e-2)


@pytest.mark.parametrize("B,S,D,H,Hkv,FF,causal", [
    (1, 64, 128, 4, 2, 256, False),    # head_dim 32
    (2, 100, 256, 4, 2, 192, True),    # head_dim 64, ragged S, causal, batch
    (1, 40, 512, 4, 1, 128, False),    # head_dim 128, one kv head
    (1, 33, 96, 2, 2, 64, True),       # head_dim 48 (not a multiple of 32)
])
def test_llama_decoder_f32_matches_oracle(B, S, D, H, Hkv, FF, causal):
    import torch
    from metalbench_b200 import ops
    rng = np.random.default_rng(S + D)
    Dh = D // H
    x = rng.standard_normal((B, S, D), dtype=np.float32)
    W = [rng.standard_normal(s, dtype=np.float32) * np.float32(0.1)
         for s in [(D, D + 2 * Hkv * Dh), (D, D), (D, 2 * FF), (FF, D)]]
    y = ops.llama_decoder_f32(_t(torch, x), *[_t(torch, w) for w in W], n_heads=H,
                              n_kv_heads=Hkv, base=10000.0, causal=causal)
    want = O.decoder_layer(x, *W, H=H, H_kv=Hkv, base=10000.0, causal=causal, acc=np.float64)
    _all_within(y.cpu().numpy(), want, 1e-2)
