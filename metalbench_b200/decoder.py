"""LLaMA decoder layer on libmb200 (torch tensors for device memory only).

Mirrors the reference hook ``mlx/kernels/full/llama_decoder_layer.py``:
``Model(S, D, H, H_kv, FF, base, eps).forward(x, W_qkv, W_o, W_gu, W_down)``,
weights in the reference (in, out) layout. ``DecoderLayer`` packs them once
(K-major, this rank's tensor-parallel shard) and runs the fused kernels;
``PagedKVCache`` holds the rotated keys and values of every sequence in
64-token pages.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib, ops

PAGE = 64


@dataclass
class DecoderConfig:
    d_model: int
    n_heads: int
    n_kv_heads: int
    ffn: int
    head_dim: int = 128
    rope_base: float = 10000.0
    eps: float = 1e-5

    def as_c(self) -> _lib.MbDecoderConfig:
        return _lib.MbDecoderConfig(self.d_model, self.n_heads, self.n_kv_heads, self.head_dim,
                                    self.ffn, float(self.rope_base), float(self.eps))


class PagedKVCache:
    """k, v: [num_pages, Hkv_local, 64, Dh] bf16; block_table [B, max_pages] int32.

    Sequence b owns pages b*max_pages .. b*max_pages+max_pages-1 (a simple
    contiguous assignment; any page permutation works with the kernels)."""

    def __init__(self, batch: int, max_len: int, n_kv_heads: int, head_dim: int = 128,
                 device=None, block_table: torch.Tensor | None = None):
        device = device or torch.device("cuda", torch.cuda.current_device())
        self.batch = batch
        self.max_pages = (max_len + PAGE - 1) // PAGE
        n_pages = batch * self.max_pages
        shape = (n_pages, n_kv_heads, PAGE, head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        if block_table is None:
            block_table = torch.arange(n_pages, dtype=torch.int32, device=device).view(
                batch, self.max_pages)
        self.block_table = block_table.to(device=device, dtype=torch.int32).contiguous()
        self.max_len = self.max_pages * PAGE

    def write_positions(self, b: int, k: torch.Tensor, v: torch.Tensor, start: int = 0) -> None:
        """Store already-rotated k, v [Hkv, L, Dh] of sequence b at start.. (test/bench set-up)."""
        L = k.shape[1]
        for p in range(start, start + L):
            pg = int(self.block_table[b, p // PAGE])
            self.k[pg, :, p % PAGE] = k[:, p - start]
            self.v[pg, :, p % PAGE] = v[:, p - start]


class DecoderLayer:
    def __init__(self, cfg: DecoderConfig, W_qkv: torch.Tensor, W_o: torch.Tensor,
                 W_gu: torch.Tensor, W_down: torch.Tensor, tp_rank: int = 0, tp_world: int = 1):
        for name, t in (("W_qkv", W_qkv), ("W_o", W_o), ("W_gu", W_gu), ("W_down", W_down)):
            ops._cuda(t, f"DecoderLayer({name})", (torch.bfloat16,))
        D, Dh = cfg.d_model, cfg.head_dim
        want = {"W_qkv": (D, D + 2 * cfg.n_kv_heads * Dh), "W_o": (D, D),
                "W_gu": (D, 2 * cfg.ffn), "W_down": (cfg.ffn, D)}
        for name, t in (("W_qkv", W_qkv), ("W_o", W_o), ("W_gu", W_gu), ("W_down", W_down)):
            if tuple(t.shape) != want[name]:
                raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {want[name]}")
        ops.init(W_qkv.device.index)
        self.cfg = cfg
        self.tp_rank, self.tp_world = tp_rank, tp_world
        self.h_kv_local = cfg.n_kv_heads // tp_world
        self.h_local = cfg.n_heads // tp_world
        h = C.c_void_p()
        _lib.call("mb_decoder_layer_create", C.byref(cfg.as_c()), W_qkv.data_ptr(), W_o.data_ptr(),
                  W_gu.data_ptr(), W_down.data_ptr(), tp_rank, tp_world, C.byref(h))
        self._h = h
        torch.cuda.synchronize()

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().mb_decoder_layer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def workspace_bytes(self, B: int, S: int, max_kv_len: int) -> int:
        return _lib.lib().mb_decoder_layer_workspace_bytes(self._h, B, S, max_kv_len)

    def forward(self, x: torch.Tensor, cache: PagedKVCache, start_pos: torch.Tensor,
                causal: bool = True, out: torch.Tensor | None = None,
                max_kv_len: int | None = None, kv_len: torch.Tensor | None = None,
                x_res32: torch.Tensor | None = None,
                y_res32: torch.Tensor | None = None,
                rstd_in: torch.Tensor | None = None,
                rstd_out: torch.Tensor | None = None) -> torch.Tensor:
        """x: [B, S, D] bf16 (or [S, D] for B = 1); start_pos: int32 [B] on the device.

        The new tokens' keys/values are appended at start_pos[b].. and attention
        reads positions 0..start_pos[b]+S-1. kv_len (= start_pos + S, int32 on
        the device) may be passed in when several layers share it. x_res32 /
        y_res32 (fp32, x's shape) carry the residual stream in fp32 between
        layers: x_res32 is this layer's input residual (x its bf16 rounding),
        y_res32 receives the fp32 output. rstd_in / rstd_out (fp32, one entry
        per token) chain the input RMSNorm factor between layers: rstd_out
        receives rsqrt(mean(y_res32^2) + eps) for the next layer, which takes
        it as rstd_in instead of computing it (rstd_out needs y_res32)."""
        squeeze = x.dim() == 2
        X = x.unsqueeze(0) if squeeze else x
        ops._cuda(X, "DecoderLayer.forward(x)", (torch.bfloat16,))
        B, S, D = X.shape
        if start_pos.dtype != torch.int32 or not start_pos.is_cuda or start_pos.numel() != B:
            raise ValueError("start_pos must be an int32 CUDA tensor with one entry per sequence")
        if kv_len is None:
            kv_len = (start_pos + S).contiguous()
        if max_kv_len is None:
            max_kv_len = int(kv_len.max().item())
        if out is None:
            out = torch.empty_like(X)
        ws_bytes = self.workspace_bytes(B, S, max_kv_len)
        ws = ops._workspace(ws_bytes, X.device)
        self._kv_len = kv_len  # keep alive until the stream has consumed it
        for nm, t in (("x_res32", x_res32), ("y_res32", y_res32)):
            if t is not None:
                ops._cuda(t, f"DecoderLayer.forward({nm})", (torch.float32,))
                if t.numel() != X.numel():
                    raise ValueError(f"{nm} must have x's shape")
        for nm, t in (("rstd_in", rstd_in), ("rstd_out", rstd_out)):
            if t is not None:
                ops._cuda(t, f"DecoderLayer.forward({nm})", (torch.float32,))
                if t.numel() != B * S:
                    raise ValueError(f"{nm} must hold one float per token")
        if rstd_out is not None and y_res32 is None:
            raise ValueError("rstd_out needs y_res32")
        _lib.call("mb_decoder_layer_forward_chain", self._h, X.data_ptr(),
                  0 if x_res32 is None else x_res32.data_ptr(),
                  0 if rstd_in is None else rstd_in.data_ptr(), out.data_ptr(),
                  0 if y_res32 is None else y_res32.data_ptr(),
                  0 if rstd_out is None else rstd_out.data_ptr(), B, S,
                  start_pos.data_ptr(), kv_len.data_ptr(), max_kv_len, cache.k.data_ptr(),
                  cache.v.data_ptr(), cache.block_table.data_ptr(), cache.max_pages,
                  1 if causal else 0, ws.data_ptr(), ws_bytes, ops._stream())
        return out[0] if squeeze else out

    __call__ = forward
