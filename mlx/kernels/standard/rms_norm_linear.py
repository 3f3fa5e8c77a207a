"""rms_norm_linear reference hook: y = rms_norm(x) @ w^T, w stored (out_dim, dim).

The norm has no gain (the reference initialises its RMSNorm weight to ones and
normalises explicitly with eps 1e-5).
"""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def __init__(self, dim=1024, out_dim=1024, eps=1e-5):
        super().__init__()
        self.dim, self.out_dim, self.eps = dim, out_dim, eps

    def forward(self, x: mx.array, w: mx.array) -> mx.array:
        inv = mx.rsqrt(mx.mean(x * x, axis=-1, keepdims=True) + self.eps)
        return (x * inv) @ w.T
