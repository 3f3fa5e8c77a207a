"""fused_qkv_projection reference hook: x @ w_qkv -> (Q | K | V) concatenated."""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def forward(self, x: mx.array, w_qkv: mx.array) -> mx.array:
        return x @ w_qkv
