"""Decode attention alone, at the per-rank shape of the bench stack at a given
tensor-parallel degree, on one GPU.

    python -m metalbench_b200.attn_decode_probe --tp 8 [--iters 20]

Per rank the stack attends B 64 sequences over KV 8193 with 64/tp query heads
and 8/tp kv heads of 128 (one paged cache of N(0,1) keys and values). The
probe launches `mb_attention_decode_bf16` (the split kernel and its combine)
`--iters` times after 3 warm-up launches, times each launch with CUDA events
on the launching stream and prints one JSON line: the median milliseconds,
the algorithmic KV bytes (2 · B · 8193 · Hkv · 128 · 2) and their rate. It is
the stand-in that makes the kernel of a TP rank profilable on one GPU.
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from metalbench_b200 import _lib, ops  # noqa: E402
from metalbench_b200.decoder import PagedKVCache  # noqa: E402


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=8)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--kv", type=int, default=8193)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    ops.init(0)
    hq, hkv = 64 // a.tp, 8 // a.tp
    cache = PagedKVCache(a.batch, a.kv + 63, hkv)
    g = torch.Generator(device="cuda").manual_seed(4)
    cache.k.normal_(generator=g)
    cache.v.normal_(generator=g)
    q = torch.randn((a.batch, hq * 128), device="cuda", generator=g).bfloat16()
    out = torch.empty_like(q)
    kvl = torch.full((a.batch,), a.kv, dtype=torch.int32, device="cuda")
    nbytes = _lib.lib().mb_attention_decode_workspace_bytes(a.batch, hq, hkv, a.kv)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    stream = ops._stream()

    def launch():
        _lib.call("mb_attention_decode_bf16", q.data_ptr(), hq * 128, cache.k.data_ptr(),
                  cache.v.data_ptr(), cache.block_table.data_ptr(), cache.max_pages,
                  kvl.data_ptr(), a.kv, a.batch, hq, hkv, 128, out.data_ptr(), hq * 128,
                  ws.data_ptr(), nbytes, stream)

    for _ in range(3):
        launch()
    torch.cuda.synchronize()
    times = []
    for _ in range(a.iters):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        launch()
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    times.sort()
    ms = times[len(times) // 2]
    kv_bytes = 2 * a.batch * a.kv * hkv * 128 * 2
    print(json.dumps({"tp": a.tp, "batch": a.batch, "kv": a.kv, "hq": hq, "hkv": hkv,
                      "median_ms": ms, "kv_bytes": kv_bytes, "gbps": kv_bytes / ms / 1e6}))


if __name__ == "__main__":
    main()
