"""numpy restatement of the reference hooks on the hot path (test infrastructure).

Every function names the reference file:line whose semantics it follows. All
arithmetic is done in ``acc`` precision (float32 by default, float64 for the
known-answer tests); bf16 tensors travel as ``uint16`` bit patterns.
"""
from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------------------
# bf16 <-> f32 as raw bit patterns (numpy has no bf16 dtype).
# ----------------------------------------------------------------------------


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns (uint16) to float32 exactly."""
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to bf16 (round-to-nearest-even), returned as uint16 bits.

    NaN inputs map to a quiet NaN. This is the IEEE rounding rule applied to the
    top 16 bits; the CUDA kernels use ``__float2bfloat16_rn`` which follows the
    same rule.
    """
    f = np.ascontiguousarray(x, dtype=np.float32)
    u = f.view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        out[nan] = np.uint16(0x7FC0)
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 -> float32."""
    return bf16_to_f32(f32_to_bf16(x))


# ----------------------------------------------------------------------------
# common set
# ----------------------------------------------------------------------------


def sqr_mm(A: np.ndarray, B: np.ndarray, acc=np.float64) -> np.ndarray:
    """C = A @ B  (mlx/kernels/common/sqr_mm.py:10-11, ``mx.matmul(A, B)``).

    Row-major operands; the result is returned in float32. ``acc=np.float64``
    gives the "true" product that the 1e-4 relative-error gate is measured
    against.
    """
    return (A.astype(acc) @ B.astype(acc)).astype(np.float32)


def transpose_2d(A: np.ndarray) -> np.ndarray:
    """B = A^T, out of place (mlx/kernels/common/transpose_2d.py:10-11).

    For a rank-3 input the last two axes are swapped (the batched variant).
    Pure data movement: the result is bit-identical to the input elements.
    """
    if A.ndim == 2:
        return np.ascontiguousarray(A.T)
    return np.ascontiguousarray(np.swapaxes(A, -1, -2))


def conv2d_nhwc(x: np.ndarray, w: np.ndarray, stride: int = 1, padding: int = 0,
                acc=np.float32) -> np.ndarray:
    """``mx.conv2d(x, w, stride, padding)`` (mlx/kernels/common/conv2d.py:7-12).

    x is NHWC (N, H, W, Cin); w is OHWI (Cout, KH, KW, Cin); the operation is a
    cross-correlation (no kernel flip), symmetric zero padding, dilation 1,
    groups 1. Output NHWC (N, H2, W2, Cout), H2 = (H + 2p - KH) // stride + 1.
    """
    N, H, W, C = x.shape
    Co, KH, KW, Ci = w.shape
    assert Ci == C, "channel mismatch"
    xp = np.pad(x.astype(acc), ((0, 0), (padding, padding), (padding, padding), (0, 0)))
    H2 = (H + 2 * padding - KH) // stride + 1
    W2 = (W + 2 * padding - KW) // stride + 1
    out = np.zeros((N, H2, W2, Co), dtype=acc)
    wa = w.astype(acc)
    for r in range(KH):
        for s in range(KW):
            patch = xp[:, r:r + stride * (H2 - 1) + 1:stride, s:s + stride * (W2 - 1) + 1:stride, :]
            out += (patch.reshape(-1, C) @ wa[:, r, s, :].T).reshape(N, H2, W2, Co)
    return out.astype(np.float32)


# ----------------------------------------------------------------------------
# full set: LLaMA decoder layer
# ----------------------------------------------------------------------------


def rms_norm(x: np.ndarray, eps: float) -> np.ndarray:
    """x * rsqrt(mean(x^2) + eps), no gain vector
    (mlx/kernels/full/llama_decoder_layer.py:48-50)."""
    v = np.mean(x * x, axis=-1, keepdims=True)
    return x / np.sqrt(v + eps)


def rope_angles(positions: np.ndarray, Dh: int, base: float, acc=np.float64):
    """cos/sin tables (len(positions), Dh/2): angle = pos * base^(-2i/Dh)
    (mlx/kernels/full/llama_decoder_layer.py:54-58)."""
    half = Dh // 2
    idx = np.arange(half, dtype=acc)
    omega = 1.0 / (acc(base) ** (2.0 * idx / Dh))
    ang = positions.astype(acc)[:, None] * omega[None, :]
    return np.cos(ang), np.sin(ang)


def rope(t: np.ndarray, positions: np.ndarray, base: float) -> np.ndarray:
    """Interleaved-pair rotary embedding on (..., S, Dh): pairs (2i, 2i+1)
    rotate by angle pos*omega_i (mlx/kernels/full/llama_decoder_layer.py:52-64)."""
    Dh = t.shape[-1]
    c, s = rope_angles(positions, Dh, base, acc=np.float64)
    c = c.astype(t.dtype)
    s = s.astype(t.dtype)
    t0 = t[..., 0::2]
    t1 = t[..., 1::2]
    out = np.empty_like(t)
    out[..., 0::2] = t0 * c - t1 * s
    out[..., 1::2] = t0 * s + t1 * c
    return out


def silu(x):
    return x / (1.0 + np.exp(-x))


def decoder_layer(x, W_qkv, W_o, W_gu, W_down, *, H: int, H_kv: int,
                  base: float = 10000.0, eps: float = 1e-5, causal: bool = False,
                  k_past=None, v_past=None, pos_offset=None, acc=np.float32,
                  return_kv: bool = False):
    """LLaMA decoder layer (mlx/kernels/full/llama_decoder_layer.py:24-46).

    Reference order: RMSNorm -> h @ W_qkv -> split q | k | v (q heads first,
    then kv heads) -> RoPE on q and k -> GQA (query head h reads kv head h // G,
    ``mx.repeat`` along the head axis, line 34) -> softmax(q k^T / sqrt(Dh))
    -> (attn @ v) heads re-interleaved to (S, D) -> @ W_o -> + x -> RMSNorm ->
    h @ W_gu, gate = first FF columns, up = the rest -> silu(gate)*up @ W_down
    -> + x.

    Backward-compatible extensions (defaults reproduce the reference hook):
      * x may be (S, D) or (B, S, D);
      * ``causal`` masks keys whose position exceeds the query's;
      * ``k_past``/``v_past`` (B, H_kv, L, Dh) are a KV cache of already-rotated
        keys and values; new tokens sit at positions ``pos_offset + arange(S)``
        (``pos_offset`` defaults to L).
    Weights are stored (in, out) as in the reference. Returns y (and the new
    rotated k, v of shape (B, H_kv, S, Dh) when ``return_kv``).
    """
    squeeze = x.ndim == 2
    X = x[None] if squeeze else x
    X = X.astype(acc)
    Bn, S, D = X.shape
    Dh = D // H
    G = H // H_kv
    FF = W_down.shape[0]
    Wqkv = W_qkv.astype(acc)
    L = 0 if k_past is None else k_past.shape[2]
    p0 = L if pos_offset is None else pos_offset
    positions = np.arange(p0, p0 + S)

    h = rms_norm(X, eps)
    qkv = h @ Wqkv                                   # (B, S, D + 2*Hkv*Dh)
    q = qkv[..., :D].reshape(Bn, S, H, Dh).transpose(0, 2, 1, 3)
    k = qkv[..., D:D + H_kv * Dh].reshape(Bn, S, H_kv, Dh).transpose(0, 2, 1, 3)
    v = qkv[..., D + H_kv * Dh:].reshape(Bn, S, H_kv, Dh).transpose(0, 2, 1, 3)
    q = rope(q, positions, base)
    k = rope(k, positions, base)
    k_new, v_new = k, v
    if k_past is not None:
        k = np.concatenate([k_past.astype(acc), k], axis=2)
        v = np.concatenate([v_past.astype(acc), v], axis=2)
    kr = np.repeat(k, G, axis=1)                     # (B, H, L+S, Dh)
    vr = np.repeat(v, G, axis=1)
    scores = (q @ kr.transpose(0, 1, 3, 2)) / np.sqrt(acc(Dh))
    if causal:
        # cached keys sit at positions 0..L-1, new keys at their own positions
        key_pos = np.concatenate([np.arange(L), positions]) if k_past is not None else positions
        mask = key_pos[None, :] > positions[:, None]
        scores = np.where(mask[None, None], -np.inf, scores)
    scores = scores - scores.max(axis=-1, keepdims=True)
    e = np.exp(scores)
    attn = e / e.sum(axis=-1, keepdims=True)
    o = (attn @ vr).transpose(0, 2, 1, 3).reshape(Bn, S, D)
    X = X + o @ W_o.astype(acc)

    h = rms_norm(X, eps)
    gu = h @ W_gu.astype(acc)
    ff = (silu(gu[..., :FF]) * gu[..., FF:]) @ W_down.astype(acc)
    Y = (X + ff).astype(np.float32)
    y = Y[0] if squeeze else Y
    if return_kv:
        return y, k_new, v_new
    return y


def decoder_stack(x, layers, **kw):
    """Apply ``decoder_layer`` once per weight tuple in ``layers``."""
    for (Wqkv, Wo, Wgu, Wdown) in layers:
        x = decoder_layer(x, Wqkv, Wo, Wgu, Wdown, **kw)
    return x


# ----------------------------------------------------------------------------
# correctness gate (harness semantics)
# ----------------------------------------------------------------------------


def allclose_report(actual, expected, rtol: float, atol: float) -> dict:
    """The reference harness gate plus the element fraction.

    ``all`` is the reference's verdict ``all(|a-b| <= atol + rtol*|b|)``
    (mlx/scripts/harness.py:26-33); ``frac_within_tol`` is the fraction of
    elements that satisfy it (the mismatch percentage of
    mlx/scripts/diff_arrays.py:55-64, inverted); ``max_err`` = max |a-b|.
    """
    a = np.asarray(actual, dtype=np.float64)
    b = np.asarray(expected, dtype=np.float64)
    if a.shape != b.shape:
        return {"all": False, "frac_within_tol": 0.0, "max_err": float("inf"), "max_rel_err": float("inf")}
    if a.size == 0:
        return {"all": True, "frac_within_tol": 1.0, "max_err": 0.0, "max_rel_err": 0.0}
    diff = np.abs(a - b)
    ok = diff <= atol + rtol * np.abs(b)
    ok &= ~np.isnan(a)
    denom = np.maximum(np.abs(b), 1e-30)
    return {"all": bool(ok.all()), "frac_within_tol": float(ok.mean()),
            "max_err": float(np.nanmax(diff)), "max_rel_err": float(np.nanmax(diff / denom))}


# ----------------------------------------------------------------------------
# standard set (sub-steps of the decoder)
# ----------------------------------------------------------------------------


def rms_norm_linear(x, w, eps=1e-5, acc=np.float64):
    """rms_norm(x) @ w.T, w stored (out_dim, dim)
    (mlx/kernels/standard/rms_norm_linear.py:8-17)."""
    xa = x.astype(acc)
    return (rms_norm(xa, eps) @ w.astype(acc).T).astype(np.float32)


def fused_add_rms_norm(x, residual, eps=1e-5, acc=np.float64):
    """RMSNorm(x + residual) with unit gain
    (mlx/kernels/standard/fused_add_rms_norm.py:6-13)."""
    return rms_norm(x.astype(acc) + residual.astype(acc), eps).astype(np.float32)


def rope_full(x, base=10000.0, acc=np.float64):
    """Interleaved-pair RoPE over the full width of x (S, D), positions 0..S-1,
    omega_i = base^(-2i/D) (mlx/kernels/standard/rope_embedding.py:14-30)."""
    return rope(x.astype(acc), np.arange(x.shape[0]), base).astype(np.float32)


def swiglu(x, w_gate, w_up, acc=np.float64):
    """silu(x @ w_gate) * (x @ w_up) (mlx/kernels/standard/swiglu.py:10-11)."""
    xa = x.astype(acc)
    return (silu(xa @ w_gate.astype(acc)) * (xa @ w_up.astype(acc))).astype(np.float32)


def sdpa(Q, K, V, acc=np.float64):
    """softmax(Q K^T / sqrt(d)) V for one head
    (mlx/kernels/standard/scaled_dot_product.py:9-14)."""
    q, k, v = Q.astype(acc), K.astype(acc), V.astype(acc)
    s = q @ k.T / np.sqrt(acc(q.shape[-1]))
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    return ((p / p.sum(axis=-1, keepdims=True)) @ v).astype(np.float32)


def llama_attention(x, W_qkv, W_o, *, H: int, H_kv: int, base: float = 10000.0,
                    acc=np.float64):
    """Grouped-query self-attention with RoPE, no mask, no cache
    (mlx/kernels/standard/llama_attention.py:22-63): qkv = x @ W_qkv; q/k/v
    heads of Dh = D/H; RoPE (pairs (2i, 2i+1), positions 0..S-1) on q and k;
    query head h uses kv head h // (H/H_kv); softmax(q k^T / sqrt(Dh)) v; @ W_o."""
    S, D = x.shape
    Dh = D // H
    qkv = x.astype(acc) @ W_qkv.astype(acc)
    q = qkv[:, :D].reshape(S, H, Dh).transpose(1, 0, 2)
    k = qkv[:, D:D + H_kv * Dh].reshape(S, H_kv, Dh).transpose(1, 0, 2)
    v = qkv[:, D + H_kv * Dh:].reshape(S, H_kv, Dh).transpose(1, 0, 2)
    pos = np.arange(S)
    q = rope(q, pos, base)
    k = rope(k, pos, base)
    g = H // H_kv
    k = np.repeat(k, g, axis=0)
    v = np.repeat(v, g, axis=0)
    sc = q @ k.transpose(0, 2, 1) / np.sqrt(acc(Dh))
    sc = sc - sc.max(axis=-1, keepdims=True)
    p = np.exp(sc)
    p = p / p.sum(axis=-1, keepdims=True)
    o = (p @ v).transpose(1, 0, 2).reshape(S, D)
    return (o @ W_o.astype(acc)).astype(np.float32)


def layer_norm(x, eps=1e-5):
    """(x - mean) / sqrt(var + eps) over the last axis, no affine, ddof 0
    (mlx/kernels/full/transformer_block.py:49-52)."""
    m = x.mean(axis=-1, keepdims=True)
    v = ((x - m) ** 2).mean(axis=-1, keepdims=True)
    return (x - m) / np.sqrt(v + eps)


def gelu(x):
    """Exact GELU x * Phi(x) = 0.5 x (1 + erf(x / sqrt 2)) (MLX nn.gelu)."""
    from scipy.special import erf
    return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))


def _mha(x, W_q, W_k, W_v, H):
    S, D = x.shape
    Dh = D // H
    q = (x @ W_q).reshape(S, H, Dh).transpose(1, 0, 2)
    k = (x @ W_k).reshape(S, H, Dh).transpose(1, 0, 2)
    v = (x @ W_v).reshape(S, H, Dh).transpose(1, 0, 2)
    sc = q @ k.transpose(0, 2, 1) / np.sqrt(x.dtype.type(Dh))
    sc = sc - sc.max(axis=-1, keepdims=True)
    p = np.exp(sc)
    p = p / p.sum(axis=-1, keepdims=True)
    return (p @ v).transpose(1, 0, 2).reshape(S, D)


def mha_attention(x, wq, wk, wv, wo, *, H: int = 4, acc=np.float64):
    """Multi-head attention, H heads of D/H, no mask (mlx/kernels/full/mha_attention.py:13-28)."""
    f = lambda a: a.astype(acc)
    return (_mha(f(x), f(wq), f(wk), f(wv), H) @ f(wo)).astype(np.float32)


def transformer_block(x, W_qkv, W_o, W_ff1, W_ff2, *, H: int, eps: float = 1e-5, acc=np.float64):
    """Pre-LN block (mlx/kernels/full/transformer_block.py:22-47):
    x1 = x + MHA(LN(x)) @ W_o with W_qkv = [Wq | Wk | Wv]; y = x1 + gelu(LN(x1) @ W_ff1) @ W_ff2."""
    x = x.astype(acc)
    D = x.shape[1]
    Wqkv = W_qkv.astype(acc)
    ln1 = layer_norm(x, eps)
    x1 = x + _mha(ln1, Wqkv[:, :D], Wqkv[:, D:2 * D], Wqkv[:, 2 * D:], H) @ W_o.astype(acc)
    ff = gelu(layer_norm(x1, eps) @ W_ff1.astype(acc)) @ W_ff2.astype(acc)
    return (x1 + ff).astype(np.float32)
