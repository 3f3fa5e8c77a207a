"""Torch-tensor front end of libmb200 (device memory and streams come from torch).

Each function validates its tensors, then calls the C-ABI entry point with raw
device pointers on torch's current stream. There is no fallback: a missing
library or a non-CUDA tensor raises.
"""
from __future__ import annotations

import torch

from . import _lib

_inited: set[int] = set()


def init(device: int | None = None) -> None:
    """mb_init for one GPU (idempotent per device)."""
    dev = torch.cuda.current_device() if device is None else int(device)
    if dev not in _inited:
        _lib.call("mb_init", dev, 0, 1, None, 0)
        _inited.add(dev)


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _cuda(t: torch.Tensor, name: str, dtypes) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name}: expected a CUDA tensor (no CPU fallback)")
    if t.dtype not in dtypes:
        raise TypeError(f"{name}: dtype {t.dtype} not in {dtypes}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous tensor")


def transpose_2d(a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out = a.T for a 2-D fp32 or bf16 tensor (bit-exact data movement)."""
    _cuda(a, "transpose_2d", (torch.float32, torch.bfloat16))
    if a.dim() != 2:
        raise ValueError("transpose_2d: expected a 2-D tensor")
    init(a.device.index)
    R, Cc = a.shape
    if out is None:
        out = torch.empty((Cc, R), dtype=a.dtype, device=a.device)
    _cuda(out, "transpose_2d(out)", (a.dtype,))
    if tuple(out.shape) != (Cc, R):
        raise ValueError("transpose_2d: out has the wrong shape")
    if a.dtype == torch.float32:
        _lib.call("mb_transpose_2d_f32", a.data_ptr(), out.data_ptr(), R, Cc, _stream())
    else:
        _lib.call("mb_transpose_batched_bf16", a.data_ptr(), out.data_ptr(), 1, R, Cc, _stream())
    return out


def transpose_batched(a: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Swap the last two axes of a [batch, rows, cols] fp32 or bf16 tensor."""
    _cuda(a, "transpose_batched", (torch.float32, torch.bfloat16))
    if a.dim() != 3:
        raise ValueError("transpose_batched: expected a 3-D tensor")
    init(a.device.index)
    Bn, R, Cc = a.shape
    if out is None:
        out = torch.empty((Bn, Cc, R), dtype=a.dtype, device=a.device)
    _cuda(out, "transpose_batched(out)", (a.dtype,))
    if tuple(out.shape) != (Bn, Cc, R):
        raise ValueError("transpose_batched: out has the wrong shape")
    fn = "mb_transpose_batched_f32" if a.dtype == torch.float32 else "mb_transpose_batched_bf16"
    _lib.call(fn, a.data_ptr(), out.data_ptr(), Bn, R, Cc, _stream())
    return out


def gemm_bf16(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
              b_layout: str = "kn") -> torch.Tensor:
    """bf16 GEMM on the tcgen05 core. ``b_layout="kn"``: b is [K, N] (a @ b);
    ``"nk"``: b is [N, K] (a @ b.T, the packed-weight layout)."""
    _cuda(a, "gemm_bf16(a)", (torch.bfloat16,))
    _cuda(b, "gemm_bf16(b)", (torch.bfloat16,))
    init(a.device.index)
    M, K = a.shape
    if b_layout == "kn":
        Kb, N = b.shape
        lay = 1
    elif b_layout == "nk":
        N, Kb = b.shape
        lay = 0
    else:
        raise ValueError("b_layout must be 'kn' or 'nk'")
    if Kb != K:
        raise ValueError(f"gemm_bf16: inner dimensions differ ({K} vs {Kb})")
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    _cuda(out, "gemm_bf16(out)", (torch.bfloat16,))
    _lib.call("mb_gemm_bf16", a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, lay, _stream())
    return out


def sqr_mm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 C = A @ B (row-major), fp32-accurate 3xTF32 on the tensor cores."""
    _cuda(a, "sqr_mm(a)", (torch.float32,))
    _cuda(b, "sqr_mm(b)", (torch.float32,))
    init(a.device.index)
    M, K = a.shape
    Kb, N = b.shape
    if Kb != K:
        raise ValueError(f"sqr_mm: inner dimensions differ ({K} vs {Kb})")
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=a.device)
    _cuda(out, "sqr_mm(out)", (torch.float32,))
    ws_bytes = _lib.lib().mb_sqr_mm_f32_workspace_bytes(M, N, K)
    ws = _workspace(ws_bytes, a.device)
    _lib.call("mb_sqr_mm_f32", a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K,
              ws.data_ptr() if ws_bytes else None, ws_bytes, _stream())
    return out


def batch_mm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """fp32 C[i] = A[i] @ B[i] for a [batch, M, K] and b [batch, K, N], 3xTF32."""
    _cuda(a, "batch_mm(a)", (torch.float32,))
    _cuda(b, "batch_mm(b)", (torch.float32,))
    init(a.device.index)
    Bt, M, K = a.shape
    Bb, Kb, N = b.shape
    if (Bb, Kb) != (Bt, K):
        raise ValueError(f"batch_mm: shapes {tuple(a.shape)} and {tuple(b.shape)} do not match")
    out = torch.empty((Bt, M, N), dtype=torch.float32, device=a.device)
    ws_bytes = _lib.lib().mb_batch_mm_f32_workspace_bytes(Bt, M, N, K)
    ws = _workspace(ws_bytes, a.device)
    _lib.call("mb_batch_mm_f32", a.data_ptr(), b.data_ptr(), out.data_ptr(), Bt, M, N, K,
              ws.data_ptr() if ws_bytes else None, ws_bytes, _stream())
    return out


_ws: dict = {}


def _workspace(nbytes: int, device) -> torch.Tensor:
    """Per-device scratch tensor, grown on demand (256-byte aligned by torch)."""
    key = device.index
    t = _ws.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
        _ws[key] = t
    return t


def conv2d_nhwc(x: torch.Tensor, w: torch.Tensor, stride: int = 1, padding: int = 0,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """NHWC x OHWI conv2d (cross-correlation). bf16: tcgen05 implicit GEMM;
    fp32: im2col + 3xTF32 GEMM (fp32-accurate, any stride / padding)."""
    _cuda(x, "conv2d(x)", (torch.bfloat16, torch.float32))
    _cuda(w, "conv2d(w)", (x.dtype,))
    init(x.device.index)
    N, H, W, C = x.shape
    Co, KH, KW, Ci = w.shape
    if Ci != C:
        raise ValueError(f"conv2d: channel mismatch ({C} vs {Ci})")
    H2 = (H + 2 * padding - KH) // stride + 1
    W2 = (W + 2 * padding - KW) // stride + 1
    if out is None:
        out = torch.empty((N, H2, W2, Co), dtype=x.dtype, device=x.device)
    _cuda(out, "conv2d(out)", (x.dtype,))
    if tuple(out.shape) != (N, H2, W2, Co):
        raise ValueError("conv2d: out has the wrong shape")
    if x.dtype == torch.float32:
        nb = _lib.lib().mb_conv2d_nhwc_f32_workspace_bytes(N, H, W, C, Co, KH, KW, stride, padding)
        if nb == 0:
            raise ValueError("conv2d: unsupported fp32 geometry (Cin must be a multiple of 4)")
        ws = _workspace(nb, x.device)
        _lib.call("mb_conv2d_nhwc_f32", x.data_ptr(), w.data_ptr(), out.data_ptr(), N, H, W, C,
                  Co, KH, KW, stride, padding, ws.data_ptr(), nb, _stream())
        return out
    _lib.call("mb_conv2d_nhwc_bf16", x.data_ptr(), w.data_ptr(), out.data_ptr(), N, H, W, C, Co,
              KH, KW, stride, padding, _stream())
    return out


def llama_decoder_f32(x: torch.Tensor, w_qkv: torch.Tensor, w_o: torch.Tensor,
                      w_gu: torch.Tensor, w_down: torch.Tensor, n_heads: int, n_kv_heads: int,
                      base: float = 10000.0, eps: float = 1e-5, causal: bool = False) -> torch.Tensor:
    """The reference decoder hook in fp32 (any even head_dim <= 256): x [S, D]
    or [B, S, D], weights (in, out) fp32; tokens at positions 0..S-1."""
    for nm, t in (("x", x), ("W_qkv", w_qkv), ("W_o", w_o), ("W_gu", w_gu), ("W_down", w_down)):
        _cuda(t, f"llama_decoder_f32({nm})", (torch.float32,))
    init(x.device.index)
    X = x.unsqueeze(0) if x.dim() == 2 else x
    B, S, D = X.shape
    FF = w_down.shape[0]
    Dh = D // n_heads
    want = {"W_qkv": (D, D + 2 * n_kv_heads * Dh), "W_o": (D, D), "W_gu": (D, 2 * FF),
            "W_down": (FF, D)}
    for nm, t in (("W_qkv", w_qkv), ("W_o", w_o), ("W_gu", w_gu), ("W_down", w_down)):
        if tuple(t.shape) != want[nm]:
            raise ValueError(f"llama_decoder_f32: {nm} has shape {tuple(t.shape)}, expected {want[nm]}")
    nb = _lib.lib().mb_llama_decoder_f32_workspace_bytes(B, S, D, n_heads, n_kv_heads, FF)
    if nb == 0:
        raise ValueError("llama_decoder_f32: unsupported geometry (head_dim even <= 256, "
                         "D and FF multiples of 4)")
    ws = _workspace(nb, x.device)
    y = torch.empty_like(X)
    _lib.call("mb_llama_decoder_f32", X.data_ptr(), w_qkv.data_ptr(), w_o.data_ptr(),
              w_gu.data_ptr(), w_down.data_ptr(), y.data_ptr(), B, S, D, n_heads, n_kv_heads, FF,
              float(base), float(eps), 1 if causal else 0, ws.data_ptr(), nb, _stream())
    return y[0] if x.dim() == 2 else y


def rms_norm_linear(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """y = rms_norm(x) @ w.T for bf16 x [M, K], w [N, K]."""
    _cuda(x, "rms_norm_linear(x)", (torch.bfloat16,))
    _cuda(w, "rms_norm_linear(w)", (torch.bfloat16,))
    init(x.device.index)
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"rms_norm_linear: w must be [N, {K}], got {tuple(w.shape)}")
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    nb = _lib.lib().mb_rms_norm_linear_workspace_bytes(M)
    ws = _workspace(nb, x.device)
    _lib.call("mb_rms_norm_linear_bf16", x.data_ptr(), w.data_ptr(), y.data_ptr(), M, K, N, eps,
              ws.data_ptr(), nb, _stream())
    return y


def fused_add_rms_norm(x: torch.Tensor, residual: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    _cuda(x, "fused_add_rms_norm(x)", (torch.bfloat16,))
    _cuda(residual, "fused_add_rms_norm(residual)", (torch.bfloat16,))
    if residual.shape != x.shape:
        raise ValueError("fused_add_rms_norm: x and residual shapes differ")
    init(x.device.index)
    y = torch.empty_like(x)
    _lib.call("mb_fused_add_rms_norm_bf16", x.data_ptr(), residual.data_ptr(), y.data_ptr(),
              x.numel() // x.shape[-1], x.shape[-1], eps, _stream())
    return y


def rope(x: torch.Tensor, base: float = 10000.0) -> torch.Tensor:
    """Interleaved-pair RoPE of x [S, D] at positions 0..S-1 over the full width."""
    _cuda(x, "rope(x)", (torch.bfloat16,))
    init(x.device.index)
    y = torch.empty_like(x)
    _lib.call("mb_rope_bf16", x.data_ptr(), y.data_ptr(), x.shape[0], x.shape[1], base, _stream())
    return y


def swiglu_pack(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    _cuda(w_gate, "swiglu_pack(w_gate)", (torch.bfloat16,))
    _cuda(w_up, "swiglu_pack(w_up)", (torch.bfloat16,))
    if w_up.shape != w_gate.shape:
        raise ValueError("swiglu_pack: w_gate and w_up shapes differ")
    init(w_gate.device.index)
    D, FF = w_gate.shape
    packed = torch.empty(_lib.lib().mb_swiglu_packed_bytes(D, FF), dtype=torch.uint8,
                         device=w_gate.device)
    _lib.call("mb_swiglu_pack_bf16", w_gate.data_ptr(), w_up.data_ptr(), packed.data_ptr(), D, FF,
              _stream())
    return packed


def swiglu(x: torch.Tensor, packed: torch.Tensor, ffn: int) -> torch.Tensor:
    """silu(x @ w_gate) * (x @ w_up) with weights from swiglu_pack."""
    _cuda(x, "swiglu(x)", (torch.bfloat16,))
    init(x.device.index)
    M, D = x.shape
    if packed.numel() < _lib.lib().mb_swiglu_packed_bytes(D, ffn):
        raise ValueError("swiglu: packed weights are smaller than swiglu_pack makes for D, ffn")
    out = torch.empty((M, ffn), dtype=torch.bfloat16, device=x.device)
    _lib.call("mb_swiglu_bf16", x.data_ptr(), packed.data_ptr(), out.data_ptr(), M, D, ffn,
              _stream())
    return out


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """softmax(q k^T / sqrt(128)) v for one head, [S, 128] bf16."""
    for n, t in (("q", q), ("k", k), ("v", v)):
        _cuda(t, f"sdpa({n})", (torch.bfloat16,))
    if not (q.shape == k.shape == v.shape) or q.dim() != 2:
        raise ValueError("sdpa: q, k, v must all be [S, 128]")
    init(q.device.index)
    S = q.shape[0]
    o = torch.empty_like(q)
    nb = _lib.lib().mb_sdpa_workspace_bytes(S)
    ws = _workspace(nb, q.device)
    _lib.call("mb_sdpa_bf16", q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), S,
              q.shape[1], ws.data_ptr(), nb, _stream())
    return o


def llama_attention(x: torch.Tensor, w_qkv: torch.Tensor, w_o: torch.Tensor, n_heads: int,
                    n_kv_heads: int, base: float = 10000.0) -> torch.Tensor:
    """GQA self-attention with RoPE over x [S, D] (bf16, head dim 128, non-causal):
    (softmax(rope(x Wq) rope(x Wk)^T / sqrt(128)) x Wv) @ W_o, weights (in, out)."""
    for n, t in (("x", x), ("w_qkv", w_qkv), ("w_o", w_o)):
        _cuda(t, f"llama_attention({n})", (torch.bfloat16,))
    init(x.device.index)
    S, D = x.shape
    out = torch.empty((S, D), dtype=torch.bfloat16, device=x.device)
    nb = _lib.lib().mb_llama_attention_workspace_bytes(S, D, n_heads, n_kv_heads)
    ws = _workspace(nb, x.device)
    _lib.call("mb_llama_attention_bf16", x.data_ptr(), w_qkv.data_ptr(), w_o.data_ptr(),
              out.data_ptr(), S, D, n_heads, n_kv_heads, base, ws.data_ptr(), nb, _stream())
    return out


def mha_attention(x: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor,
                  wo: torch.Tensor) -> torch.Tensor:
    """Multi-head self-attention of x [S, D] with heads of 128 (bf16, no mask,
    no RoPE), weights (in, out) [D, D]."""
    for n, t in (("x", x), ("wq", wq), ("wk", wk), ("wv", wv), ("wo", wo)):
        _cuda(t, f"mha_attention({n})", (torch.bfloat16,))
    init(x.device.index)
    S, D = x.shape
    out = torch.empty((S, D), dtype=torch.bfloat16, device=x.device)
    nb = _lib.lib().mb_mha_attention_workspace_bytes(S, D)
    ws = _workspace(nb, x.device)
    _lib.call("mb_mha_attention_bf16", x.data_ptr(), wq.data_ptr(), wk.data_ptr(), wv.data_ptr(),
              wo.data_ptr(), out.data_ptr(), S, D, ws.data_ptr(), nb, _stream())
    return out


def transformer_block(x: torch.Tensor, w_qkv: torch.Tensor, w_o: torch.Tensor,
                      w_ff1: torch.Tensor, w_ff2: torch.Tensor, n_heads: int,
                      eps: float = 1e-5) -> torch.Tensor:
    """Pre-LN block y = x1 + gelu(LN(x1) W_ff1) W_ff2, x1 = x + MHA(LN(x)) W_o
    (bf16, heads of 128, weights (in, out))."""
    for n, t in (("x", x), ("w_qkv", w_qkv), ("w_o", w_o), ("w_ff1", w_ff1), ("w_ff2", w_ff2)):
        _cuda(t, f"transformer_block({n})", (torch.bfloat16,))
    init(x.device.index)
    S, D = x.shape
    FF = w_ff1.shape[1]
    out = torch.empty((S, D), dtype=torch.bfloat16, device=x.device)
    nb = _lib.lib().mb_transformer_block_workspace_bytes(S, D, n_heads, FF)
    ws = _workspace(nb, x.device)
    _lib.call("mb_transformer_block_bf16", x.data_ptr(), w_qkv.data_ptr(), w_o.data_ptr(),
              w_ff1.data_ptr(), w_ff2.data_ptr(), out.data_ptr(), S, D, n_heads, FF, eps,
              ws.data_ptr(), nb, _stream())
    return out
