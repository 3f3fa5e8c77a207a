"""mha_attention reference hook: multi-head self-attention with four separate
(in, out) projections; x (S, D), wq/wk/wv/wo (D, D), 4 heads of D/4, scores
scaled by 1/sqrt(D/4), no mask, no positional rotation."""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def __init__(self, n_heads=4):
        super().__init__()
        self.n_heads = n_heads

    def forward(self, x, wq, wk, wv, wo):
        S, D = x.shape
        H = self.n_heads
        Dh = D // H

        def split(t):  # (S, D) -> (H, S, Dh)
            return t.reshape(S, H, Dh).transpose(1, 0, 2)

        q, k, v = split(x @ wq), split(x @ wk), split(x @ wv)
        w = mx.softmax((q @ k.transpose(0, 2, 1)) * (1.0 / mx.sqrt(mx.array(float(Dh)))), axis=-1)
        return (w @ v).transpose(1, 0, 2).reshape(S, D) @ wo
