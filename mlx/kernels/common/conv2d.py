"""conv2d reference hook: NHWC input x, OHWI weight w (cross-correlation).

Constructor arguments match the reference hook (in_channels, out_channels,
kernel_size, stride); ``padding`` (default 0, the reference's fixed value) is a
backward-compatible addition for the pad-1 benchmark configuration.
"""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def __init__(self, in_channels=64, out_channels=128, kernel_size=3, stride=1, padding=0):
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = kernel_size
        self.stride = stride
        self.padding = padding

    def forward(self, x: mx.array, w: mx.array) -> mx.array:
        return mx.conv2d(x, w, stride=self.stride, padding=self.padding, dilation=1, groups=1)
