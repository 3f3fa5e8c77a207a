"""fused_add_rms_norm reference hook: y = rms_norm(x + residual), unit gain."""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def __init__(self, dim: int = 1024, eps: float = 1e-5):
        super().__init__()
        self.dim, self.eps = dim, eps

    def forward(self, x: mx.array, residual: mx.array) -> mx.array:
        h = x + residual
        return h * mx.rsqrt(mx.mean(h * h, axis=-1, keepdims=True) + self.eps)
