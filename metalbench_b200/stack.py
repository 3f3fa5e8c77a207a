"""Multi-layer LLaMA decoder stack, tensor-parallel over one process per GPU.

Megatron-style sharding inside every layer (libmb200 packs each rank's shard):
q/k/v heads and gate/up features are split by column, o-proj and down-proj by
row, and their two partial outputs per layer are summed by an NCCL all-reduce
over NVLink inside ``mb_decoder_layer_forward_ex``; the residual stream is
handed from layer to layer in fp32. The KV cache holds only this rank's kv
heads. A decode step (one new token for each of B sequences
through every layer) can be captured once in a CUDA graph and replayed.
"""
from __future__ import annotations

import os
import uuid

import torch

from . import _lib, ops
from .decoder import DecoderConfig, DecoderLayer, PagedKVCache

_tp_ready = False


def init_tensor_parallel(rank: int, world: int, local_rank: int, timeout_ms: int = 120000) -> None:
    """Create libmb200's NCCL communicator (needs torch.distributed initialised:
    rank 0 picks a fresh rendezvous file name and broadcasts it)."""
    global _tp_ready
    if world == 1 or _tp_ready:
        ops.init(local_rank)
        return
    import torch.distributed as dist
    names = [os.path.join("/tmp", f"mb200_nccl_{uuid.uuid4().hex}.id") if rank == 0 else None]
    dist.broadcast_object_list(names, src=0)
    _lib.call("mb_init", local_rank, rank, world, names[0].encode(), timeout_ms)
    ops._inited.add(local_rank)
    _tp_ready = True
    dist.barrier()
    if rank == 0:
        try:
            os.unlink(names[0])
        except OSError:
            pass


class DecoderStack:
    """``n_layers`` decoder layers with random N(0, std) weights (seeded per
    layer, identical on every rank) and one paged KV cache per layer."""

    def __init__(self, cfg: DecoderConfig, n_layers: int, batch: int, max_len: int,
                 tp_rank: int = 0, tp_world: int = 1, seed: int = 4, std: float = 0.02,
                 weights=None):
        self.cfg, self.n_layers, self.batch = cfg, n_layers, batch
        self.tp_rank, self.tp_world = tp_rank, tp_world
        self.layers: list[DecoderLayer] = []
        self.caches: list[PagedKVCache] = []
        D, Dh, Hkv, FF = cfg.d_model, cfg.head_dim, cfg.n_kv_heads, cfg.ffn
        dev = torch.device("cuda", torch.cuda.current_device())
        for i in range(n_layers):
            if weights is not None:
                W = weights[i]
            else:
                g = torch.Generator(device=dev).manual_seed(seed * 1000 + i)
                W = [torch.randn(s, generator=g, device=dev, dtype=torch.bfloat16) * std
                     for s in [(D, D + 2 * Hkv * Dh), (D, D), (D, 2 * FF), (FF, D)]]
            self.layers.append(DecoderLayer(cfg, *W, tp_rank=tp_rank, tp_world=tp_world))
            del W
            self.caches.append(PagedKVCache(batch, max_len, Hkv // tp_world, Dh, device=dev))
        torch.cuda.empty_cache()
        self._graph = None

    def fill_cache_random(self, length: int, seed: int = 4) -> None:
        """Fill positions 0..length-1 of every cache with N(0,1) keys/values
        (stand-in for an already-processed prompt)."""
        g = torch.Generator(device=self.caches[0].k.device).manual_seed(seed + 7919 * self.tp_rank)
        for c in self.caches:
            c.k.normal_(generator=g)
            c.v.normal_(generator=g)

    def forward(self, x: torch.Tensor, start_pos: torch.Tensor, causal: bool = True,
                kv_len_max: int | None = None) -> torch.Tensor:
        # one kv_len for all layers: no extra kernel between two layers' launches
        S = x.shape[-2] if x.dim() == 3 else x.shape[0]
        self._kv_len = (start_pos + S).contiguous()
        # the residual stream stays fp32 from layer to layer (two ping-pong
        # buffers); each layer also emits the bf16 copy the next one's GEMMs read
        key = tuple(x.shape)
        if getattr(self, "_res_key", None) != key:
            self._res = [torch.empty(key, dtype=torch.float32, device=x.device) for _ in range(2)]
            # each layer hands the next its input RMSNorm factor (one per token)
            self._rstd = [torch.empty(key[:-1], dtype=torch.float32, device=x.device)
                          for _ in range(2)]
            self._res_key = key
        res, rstd = None, None
        last = len(self.layers) - 1
        for i, (layer, cache) in enumerate(zip(self.layers, self.caches)):
            nxt = self._res[i % 2]
            nrstd = self._rstd[i % 2] if i < last else None
            x = layer(x, cache, start_pos, causal=causal, max_kv_len=kv_len_max,
                      kv_len=self._kv_len, x_res32=res, y_res32=nxt, rstd_in=rstd,
                      rstd_out=nrstd)
            res, rstd = nxt, nrstd
        return x

    # ---- decode step in a CUDA graph ---------------------------------------
    def capture_decode(self, x: torch.Tensor, start_pos: torch.Tensor, kv_len_max: int) -> None:
        """Record one decode step (x [B, 1, D] -> self.graph_out) in a CUDA graph.
        Buffers x and start_pos are captured by address: update them in place."""
        self._gx, self._gsp = x, start_pos
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):  # warm: sets kernel attributes, sizes the workspace
                self.forward(x, start_pos, kv_len_max=kv_len_max)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.graph_out = self.forward(x, start_pos, kv_len_max=kv_len_max)
        self._graph = g

    def replay(self) -> torch.Tensor:
        self._graph.replay()
        return self.graph_out

    def close(self):
        self._graph = None
        for layer in self.layers:
            layer.close()
