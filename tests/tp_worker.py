"""Worker for the multi-GPU parity tests (launched by tests/test_tp_gpu.py with
torchrun, one process per GPU; world 1 runs the same code on one GPU).

    python -m torch.distributed.run --nproc-per-node N tests/tp_worker.py MODE

Modes:
  small  a decoder layer (D 1024, 8 query heads) sharded over the ranks,
         causal prefill then one decode step, against the oracle.
  geom   the bench's head geometry: 64 query / 8 kv heads of 128 (G = 8 query
         heads per kv head, one kv head per rank at 8 GPUs), D 8192, a reduced
         FFN of 2048; prefill then decode, against the oracle.
  stack  the bench's own workload (8-layer stack, d 8192, 64/8 heads, FFN
         28672, batch 64, KV 8192, weights N(0,0.02) seed 4, random cache),
         one decode step replayed from its CUDA graph; sequences 0..3 are
         checked against the oracle run layer by layer on the same weights and
         cache contents (gathered from every rank's kv-head shard); like the
         reference the oracle keeps the residual stream in fp32, as the stack
         does between its layers.
  gemm   the sharded bf16 GEMM 16384^3 (A, B ~ N(0,1) seed 4, B column-sharded):
         every rank checks 32 sampled rows of its column block of C against a
         float64 product.

Gate (the north-star bf16 bar, reference semantics mlx/scripts/harness.py:26-33
with a bf16 tolerance): >= 99 % of elements within 2e-2*|b| + 2e-2*rms(b), and
max |a-b| <= 0.1*rms(b). Exit code 0 = every rank passed; each rank prints one
``[mode/world/rank] ...`` line.
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import oracle.ops as O  # noqa: E402
from metalbench_b200.decoder import DecoderConfig, DecoderLayer, PagedKVCache  # noqa: E402
from metalbench_b200.stack import DecoderStack, init_tensor_parallel  # noqa: E402


def gate(got, ref):
    rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    rep = O.allclose_report(got, ref, rtol=2e-2, atol=2e-2 * rms)
    err = np.abs(got.astype(np.float64) - ref)
    mx = float(err.max())
    ok = rep["frac_within_tol"] >= 0.99 and mx <= 0.1 * rms
    i = int(err.argmax())
    return ok, {"frac": rep["frac_within_tol"], "max_abs": mx, "rms": rms,
                "rel_l2": float(np.sqrt((err ** 2).sum() / (ref.astype(np.float64) ** 2).sum())),
                "err_std": float(err.std()), "ref_at_max": float(ref.flat[i]),
                "frac_at_4e-2rms": float(np.mean(err <= 2e-2 * np.abs(ref) + 4e-2 * rms))}


def to_np(t):
    return O.bf16_to_f32(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def bf(a):
    return torch.from_numpy(O.f32_to_bf16(a).view(np.int16)).cuda().view(torch.bfloat16)


def layer_prefill_decode(rank, world, D, H, Hkv, FF, B, S, seed):
    """Prefill S tokens then decode one, sharded; returns (ok, info, out)."""
    rng = np.random.default_rng(seed)
    base = 500000.0
    r = lambda *s: O.round_bf16((rng.standard_normal(s) * 0.02).astype(np.float32))
    W = [r(D, D + 2 * Hkv * 128), r(D, D), r(D, 2 * FF), r(FF, D)]
    x = O.round_bf16(rng.standard_normal((B, S + 1, D)).astype(np.float32))
    layer = DecoderLayer(DecoderConfig(D, H, Hkv, FF, rope_base=base), *[bf(w) for w in W],
                         tp_rank=rank, tp_world=world)
    cache = PagedKVCache(B, S + 64, Hkv // world)
    y0 = layer(bf(x[:, :S]), cache, torch.zeros(B, dtype=torch.int32, device="cuda"))
    y1 = layer(bf(x[:, S:]), cache, torch.full((B,), S, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    got = np.concatenate([to_np(y0), to_np(y1)], axis=1)
    ok, info = True, {}
    if rank == 0:
        ref = O.decoder_layer(x, *W, H=H, H_kv=Hkv, base=base, causal=True)
        ok, info = gate(got, ref)
    layer.close()
    return ok, info, got


def mode_small(rank, world):
    return layer_prefill_decode(rank, world, 1024, 8, 4 if world <= 4 else 8, 1024, 2, 96, 11)


def mode_geom(rank, world):
    return layer_prefill_decode(rank, world, 8192, 64, 8, 2048, 2, 65, 12)


def gather_subset_cache(cache, seqs, L, world):
    """K, V of sequences `seqs` at positions 0..L-1, all kv heads, as float32
    arrays [len(seqs), Hkv, L, 128] on rank 0 (None elsewhere)."""
    mp = cache.max_pages
    parts = []
    for t in (cache.k, cache.v):
        rows = torch.stack([t[b * mp:b * mp + L // 64] for b in seqs])  # [n, L/64, hk, 64, 128]
        rows = rows.permute(0, 2, 1, 3, 4).reshape(len(seqs), t.shape[1], L, 128).contiguous()
        if world > 1:
            allr = [torch.empty_like(rows) for _ in range(world)]
            dist.all_gather(allr, rows)
            rows = torch.cat(allr, dim=1)  # rank r holds kv heads r*hk .. (r+1)*hk-1
        parts.append(to_np(rows) if dist.get_rank() == 0 else None)
    return parts


def mode_stack(rank, world):
    """The bench's decoder_stack workload, checked on sequences 0..3."""
    B, L, LAYERS = 64, 8192, 8
    D, H, HKV, FF = 8192, 64, 8, 28672
    base, std, seed = 500000.0, 0.02, 4
    cfg = DecoderConfig(D, H, HKV, FF, rope_base=base)
    st = DecoderStack(cfg, LAYERS, B, L + 64, tp_rank=rank, tp_world=world, seed=seed, std=std)
    st.fill_cache_random(L)
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn((B, 1, D), generator=g, device="cuda").bfloat16()
    sp = torch.full((B,), L, dtype=torch.int32, device="cuda")
    st.capture_decode(x, sp, L + 1)
    # the captured warm-ups wrote position L already; the replay rewrites it
    y = st.replay()
    torch.cuda.synchronize()
    got = to_np(y)
    seqs = [0, 1, 2, 3]
    caches = [gather_subset_cache(c, seqs, L, world) for c in st.caches]
    ok, info = True, {}
    if rank == 0:
        h = to_np(x[seqs])  # (4, 1, D)
        dev = torch.device("cuda", torch.cuda.current_device())
        Dh = 128
        for i in range(LAYERS):
            gw = torch.Generator(device=dev).manual_seed(seed * 1000 + i)
            W = [to_np(torch.randn(s, generator=gw, device=dev, dtype=torch.bfloat16) * std)
                 for s in [(D, D + 2 * HKV * Dh), (D, D), (D, 2 * FF), (FF, D)]]
            kp, vp = caches[i]
            h = O.decoder_layer(h, *W, H=H, H_kv=HKV, base=base, causal=True, k_past=kp,
                                v_past=vp)
            del W
        ok, info = gate(got[seqs], h)
        info["seqs"] = seqs
    st.close()
    return ok, info, got


def mode_gemm(rank, world):
    """Sharded 16384^3 bf16 GEMM as bench.py's gemm workload runs it."""
    from metalbench_b200 import ops
    M = N = K = 16384
    nloc = N // world
    g = torch.Generator(device="cuda").manual_seed(4)
    a = torch.randn((M, K), generator=g, device="cuda").bfloat16()
    b = torch.randn((K, N), generator=g, device="cuda").bfloat16()
    b = b[:, rank * nloc:(rank + 1) * nloc].contiguous()
    torch.cuda.empty_cache()
    c = torch.empty((M, nloc), device="cuda", dtype=torch.bfloat16)
    ops.gemm_bf16(a, b, c, b_layout="kn")
    torch.cuda.synchronize()
    rows = np.random.default_rng(100 + rank).choice(M, 32, replace=False)
    rows.sort()
    idx = torch.from_numpy(rows).cuda()
    A = to_np(a[idx]).astype(np.float64)
    Bm = to_np(b).astype(np.float64)
    ref = A @ Bm
    got = to_np(c[idx])
    ok, info = gate(got, ref)
    info["rows"] = len(rows)
    info["cols"] = f"{rank * nloc}..{(rank + 1) * nloc - 1}"
    return ok, info, None


MODES = {"small": mode_small, "geom": mode_geom, "stack": mode_stack, "gemm": mode_gemm}


def main():
    mode = sys.argv[1] if len(sys.argv) > 1 else "small"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    init_tensor_parallel(rank, world, local)
    ok, info, got = MODES[mode](rank, world)
    same = True
    if got is not None and world > 1:
        # every rank must hold the same all-reduced output
        t = torch.from_numpy(got).cuda()
        t0 = t.clone()
        dist.broadcast(t0, 0)
        same = bool(torch.equal(t, t0))
    print(f"[{mode}/world{world}/rank{rank}] ok={ok} ranks_identical={same} {info}", flush=True)
    flags = torch.tensor([int(ok and same)], device="cuda")
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    sys.exit(0 if flags.item() == 1 else 1)


if __name__ == "__main__":
    main()
