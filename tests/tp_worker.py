"""Worker for the tensor-parallel GPU test (launched by tests/test_tp_gpu.py
with torchrun, one process per GPU). Runs a small decoder layer sharded over
the ranks (prefill then decode) and checks rank 0's output against the
oracle. Exit code 0 = parity."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import oracle.ops as O  # noqa: E402
from metalbench_b200.decoder import DecoderConfig, DecoderLayer, PagedKVCache  # noqa: E402
from metalbench_b200.stack import init_tensor_parallel  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    init_tensor_parallel(rank, world, local)
    rng = np.random.default_rng(11)
    B, S, D, H, Hkv, FF, base = 2, 96, 1024, 8, 4 if world <= 4 else 8, 1024, 500000.0
    r = lambda *s: O.round_bf16((rng.standard_normal(s) * 0.02).astype(np.float32))
    W = [r(D, D + 2 * Hkv * 128), r(D, D), r(D, 2 * FF), r(FF, D)]
    x = O.round_bf16(rng.standard_normal((B, S + 1, D)).astype(np.float32))
    bf = lambda a: torch.from_numpy(O.f32_to_bf16(a).view(np.int16)).cuda().view(torch.bfloat16)
    layer = DecoderLayer(DecoderConfig(D, H, Hkv, FF, rope_base=base), *[bf(w) for w in W],
                         tp_rank=rank, tp_world=world)
    cache = PagedKVCache(B, 192, Hkv // world)
    y0 = layer(bf(x[:, :S]), cache, torch.zeros(B, dtype=torch.int32, device="cuda"))
    y1 = layer(bf(x[:, S:]), cache, torch.full((B,), S, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    to_np = lambda t: O.bf16_to_f32(t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16))
    got = np.concatenate([to_np(y0), to_np(y1)], axis=1)
    ok = True
    if rank == 0:
        ref = O.decoder_layer(x, *W, H=H, H_kv=Hkv, base=base, causal=True)
        rms = float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
        rep = O.allclose_report(got, ref, rtol=2e-2, atol=2e-2 * rms)
        ok = rep["frac_within_tol"] >= 0.99 and np.abs(got - ref).max() <= 0.1 * rms
        print(f"[tp{world}] parity {rep} ok={ok}", flush=True)
    # every rank must hold the same all-reduced output
    t = torch.from_numpy(got).cuda()
    t0 = t.clone()
    dist.broadcast(t0, 0)
    same = bool(torch.equal(t, t0))
    flags = torch.tensor([int(ok and same)], device="cuda")
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    sys.exit(0 if flags.item() == 1 else 1)


if __name__ == "__main__":
    main()
