"""llama_attention reference hook: grouped-query self-attention with RoPE and
no KV cache. x (S, D), W_qkv (D, D + 2*H_kv*Dh) packing [Wq | Wk | Wv], W_o
(D, D); H query heads share H_kv key/value heads (query head h reads kv head
h // (H / H_kv)); RoPE rotates the (2i, 2i+1) pairs of every q and k head by
pos * base^(-2i/Dh); scores are scaled by 1/sqrt(Dh) and not masked."""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def __init__(self, S=64, D=128, H=4, H_kv=2, base=10000.0):
        super().__init__()
        self.S, self.D, self.H, self.H_kv, self.base = S, D, H, H_kv, base
        self.Dh = D // H

    def _heads(self, t, n):  # (S, n*Dh) -> (n, S, Dh)
        return t.reshape(self.S, n, self.Dh).transpose(1, 0, 2)

    def _rotate(self, t):
        n, S, Dh = t.shape
        i = mx.arange(Dh // 2, dtype=mx.float32)
        inv_freq = 1.0 / (self.base ** (2.0 * i / Dh))
        theta = mx.arange(S, dtype=mx.float32)[:, None] * inv_freq[None, :]
        c, s = mx.cos(theta), mx.sin(theta)
        pairs = t.reshape(n, S, Dh // 2, 2)
        even, odd = pairs[..., 0], pairs[..., 1]
        return mx.stack([even * c - odd * s, even * s + odd * c], axis=-1).reshape(n, S, Dh)

    def forward(self, x, W_qkv, W_o):
        D, H, Hkv, Dh = self.D, self.H, self.H_kv, self.Dh
        qkv = x @ W_qkv
        q = self._rotate(self._heads(qkv[:, :D], H))
        k = self._rotate(self._heads(qkv[:, D:D + Hkv * Dh], Hkv))
        v = self._heads(qkv[:, D + Hkv * Dh:], Hkv)
        group = H // Hkv
        k, v = mx.repeat(k, group, axis=0), mx.repeat(v, group, axis=0)
        att = mx.softmax((q @ k.transpose(0, 2, 1)) / mx.sqrt(mx.array(float(Dh))), axis=-1)
        o = (att @ v).transpose(1, 0, 2).reshape(self.S, D)
        return o @ W_o
