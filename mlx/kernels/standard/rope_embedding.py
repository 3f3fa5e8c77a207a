"""rope_embedding reference hook: interleaved-pair rotary embedding of x (S, D)
at positions 0..S-1 with omega_i = base^(-2i/D) over the full width."""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def __init__(self, base: float = 10000.0):
        super().__init__()
        self.base = base

    def forward(self, x: mx.array) -> mx.array:
        S, D = x.shape
        i = mx.arange(D // 2, dtype=mx.float32)
        inv_freq = 1.0 / (self.base ** (2.0 * i / D))
        ang = mx.arange(S, dtype=mx.float32)[:, None] * inv_freq[None, :]
        cos, sin = mx.cos(ang), mx.sin(ang)
        pairs = x.reshape(S, D // 2, 2)
        even, odd = pairs[..., 0], pairs[..., 1]
        return mx.stack([even * cos - odd * sin, even * sin + odd * cos], axis=-1).reshape(S, D)
