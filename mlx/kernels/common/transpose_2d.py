"""transpose_2d reference hook: out = A with its last two axes swapped.

For a 2-D A this is A^T, the reference's mx.transpose(A)
(mlx/kernels/common/transpose_2d.py). A 3-D input [batch, rows, cols] is the
batched variant that swaps the last two axes of every matrix.
"""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def forward(self, A: mx.array) -> mx.array:
        return mx.swapaxes(A, -1, -2)
