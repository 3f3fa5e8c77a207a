"""swiglu reference hook: silu(x @ w_gate) * (x @ w_up), weights (in, out)."""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def forward(self, x: mx.array, w_gate: mx.array, w_up: mx.array) -> mx.array:
        return nn.silu(x @ w_gate) * (x @ w_up)
