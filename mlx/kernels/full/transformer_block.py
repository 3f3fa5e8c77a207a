"""transformer_block reference hook: pre-LN encoder block,
y = x1 + gelu(LN(x1) @ W_ff1) @ W_ff2 with x1 = x + MHA(LN(x)) @ W_o, where
MHA uses W_qkv = [Wq | Wk | Wv] (D, 3D) and H heads of D/H (no mask), LN
normalises each row to zero mean / unit variance (no affine), and gelu is the
exact x * Phi(x)."""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def __init__(self, S=64, D=128, H=4, FF=256, eps=1e-5):
        super().__init__()
        self.S, self.D, self.H, self.FF, self.eps = S, D, H, FF, eps

    def _ln(self, t):
        mu = mx.mean(t, axis=-1, keepdims=True)
        return (t - mu) * mx.rsqrt(mx.var(t, axis=-1, keepdims=True) + self.eps)

    def forward(self, x, W_qkv, W_o, W_ff1, W_ff2):
        S, D, H = self.S, self.D, self.H
        Dh = D // H
        qkv = self._ln(x) @ W_qkv
        q, k, v = (qkv[:, j * D:(j + 1) * D].reshape(S, H, Dh).transpose(1, 0, 2)
                   for j in range(3))
        w = mx.softmax((q @ k.transpose(0, 2, 1)) / mx.sqrt(mx.array(float(Dh))), axis=-1)
        x1 = x + (w @ v).transpose(1, 0, 2).reshape(S, D) @ W_o
        return x1 + nn.gelu(self._ln(x1) @ W_ff1) @ W_ff2
