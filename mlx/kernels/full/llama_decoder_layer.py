"""llama_decoder_layer reference hook (CPU side of ./bench llama_decoder_layer).

Contract of the reference's mlx/kernels/full/llama_decoder_layer.py:
``Model(S, D, H, H_kv, FF, base, eps).forward(x, W_qkv, W_o, W_gu, W_down)``
with weights stored (in, out): RMSNorm without gain -> x @ W_qkv -> q | k | v
(q heads, then kv heads) -> interleaved-pair RoPE (pairs 2i, 2i+1, frequency
base^(-2i/Dh)) on q and k -> query head h reads kv head h // (H/H_kv) ->
softmax(q k^T / sqrt(Dh)) @ v -> @ W_o + x -> RMSNorm -> x @ W_gu, gate = the
first FF columns -> silu(gate) * up @ W_down + residual.

Backward-compatible additions (defaults reproduce the reference):
  * x may be (B, S, D) as well as (S, D);
  * ``causal=True`` masks keys at positions after the query's;
  * ``forward(..., k_past, v_past)``: a cache (B, H_kv, L, Dh) of already-rotated
    keys / values at positions 0..L-1; the new tokens sit at positions L.. .
"""
import mlx.core as mx
from mlx import nn


class Model(nn.Module):
    def __init__(self, S=64, D=128, H=4, H_kv=2, FF=256, base=10000.0, eps=1e-5, causal=False):
        super().__init__()
        self.S, self.D, self.H, self.H_kv, self.FF = S, D, H, H_kv, FF
        self.base, self.eps, self.causal = base, eps, causal
        self.Dh = D // H
        self.group = H // H_kv

    def forward(self, x, W_qkv, W_o, W_gu, W_down, k_past=None, v_past=None):
        single = len(x.shape) == 2
        if single:
            x = x.reshape(1, *x.shape)
        B, S, D = x.shape
        H, Hkv, Dh = self.H, self.H_kv, self.Dh
        L = 0 if k_past is None else k_past.shape[2]

        # attention block
        qkv = self._norm(x) @ W_qkv
        q = qkv[..., :D].reshape(B, S, H, Dh).transpose(0, 2, 1, 3)
        k = qkv[..., D:D + Hkv * Dh].reshape(B, S, Hkv, Dh).transpose(0, 2, 1, 3)
        v = qkv[..., D + Hkv * Dh:].reshape(B, S, Hkv, Dh).transpose(0, 2, 1, 3)
        q = self._rotate(q, L)
        k = self._rotate(k, L)
        if k_past is not None:
            k = mx.concatenate([k_past, k], axis=2)
            v = mx.concatenate([v_past, v], axis=2)
        k = mx.repeat(k, self.group, axis=1)
        v = mx.repeat(v, self.group, axis=1)
        scores = (q @ k.transpose(0, 1, 3, 2)) / mx.sqrt(mx.array(float(Dh)))
        if self.causal:
            qpos = mx.arange(L, L + S)
            kpos = mx.arange(L + S)
            scores = mx.where(kpos[None, :] > qpos[:, None], mx.array(float("-inf")), scores)
        heads = mx.softmax(scores, axis=-1) @ v
        x = x + heads.transpose(0, 2, 1, 3).reshape(B, S, D) @ W_o

        # SwiGLU block
        gu = self._norm(x) @ W_gu
        y = x + (nn.silu(gu[..., :self.FF]) * gu[..., self.FF:]) @ W_down
        return y[0] if single else y

    def _norm(self, t):
        return t * mx.rsqrt(mx.mean(t * t, axis=-1, keepdims=True) + self.eps)

    def _rotate(self, t, offset):
        """RoPE on (B, heads, S, Dh) at positions offset.. offset+S-1."""
        B, nh, S, Dh = t.shape
        i = mx.arange(Dh // 2, dtype=mx.float32)
        inv_freq = 1.0 / (self.base ** (2.0 * i / Dh))
        ang = mx.arange(offset, offset + S, dtype=mx.float32)[:, None] * inv_freq[None, :]
        cos, sin = mx.cos(ang), mx.sin(ang)
        pairs = t.reshape(B, nh, S, Dh // 2, 2)
        even, odd = pairs[..., 0], pairs[..., 1]
        return mx.stack([even * cos - odd * sin, even * sin + odd * cos], axis=-1).reshape(
            B, nh, S, Dh)
