"""sqr_mm reference hook: C = A @ B for square fp32 matrices (row-major).

Same contract as the reference's mlx/kernels/common/sqr_mm.py (Model().forward(A, B)).
"""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    """Dense square matrix product."""

    def forward(self, A: mx.array, B: mx.array) -> mx.array:
        return mx.matmul(A, B)
