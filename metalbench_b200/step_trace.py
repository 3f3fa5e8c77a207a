"""Per-kernel device time of one decode step of the bench stack (CUDA-activity trace).

    python -m torch.distributed.run --nnodes=1 --master-addr=127.0.0.1 \\
        --nproc-per-node=N -m metalbench_b200.step_trace     # from the repository root

Warms the stack up (5 steps), traces 3 steps with torch.profiler and prints,
on rank 0, the kernel time per step and each kernel's launches and share.
Set MB_NO_PDL=1 so that kernels do not overlap and the shares add up. With
more than one rank, time a kernel spends waiting for the other ranks counts
as that kernel's time.
"""
import collections
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.getcwd())
import bench  # noqa: E402


def main():
    rank, world, local = bench.dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from metalbench_b200 import ops
    ops.init(local)
    wl = bench.DecoderStackDecode()
    wl.setup(torch, rank, world, local)
    for _ in range(5):
        wl.step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    steps = 3
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA],
                                acc_events=True) as prof:
        for _ in range(steps):
            wl.step()
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    for e in prof.events():
        if getattr(e, "device_type", None) is None or "cuda" not in str(e.device_type).lower():
            continue
        agg[e.name[:90]][0] += 1
        agg[e.name[:90]][1] += e.device_time_total
    tot = sum(v[1] for v in agg.values())
    if rank == 0:
        print(f"world {world}: total kernel time per step {tot / steps / 1000:.3f} ms")
        for name, (cnt, t) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
            print(f"{t / steps:10.1f} us/step {cnt / steps:6.1f} launches/step "
                  f"{100 * t / tot:5.1f}%  {name}")
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
