"""Multi-GPU parity (NVLink peer-memory reduce, NCCL for set-up and prefill) against the oracle, one process per GPU.

Each case runs tests/tp_worker.py MODE under torchrun with `world` processes
and is skipped when fewer GPUs are visible. The world-1 cases run the same
workloads unsharded on one GPU:
  * small / geom: a tensor-parallel decoder layer (prefill + decode); geom has
    the bench's 64/8 head geometry (one kv head per rank at 8 GPUs);
  * stack: the bench's 8-layer d 8192 decode step (graph replay) at full size,
    sequences 0..3 against the oracle;
  * gemm: the column-sharded 16384^3 bf16 GEMM, sampled rows of every rank's
    block against a float64 product.
"""
import os
import subprocess
import sys

import pytest

pytestmark = [pytest.mark.gpu]
HERE = os.path.dirname(os.path.abspath(__file__))

CASES = [("geom", 1), ("stack", 1), ("gemm", 1),
         ("small", 2), ("geom", 2), ("stack", 2), ("gemm", 2),
         ("small", 4), ("geom", 4), ("stack", 4),
         ("small", 8), ("geom", 8), ("stack", 8), ("gemm", 8)]


def _ngpus():
    import torch
    return torch.cuda.device_count()


def run_worker(mode, world, port=29533):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(HERE, "tp_worker.py"), mode]
    return subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900)


@pytest.mark.parametrize("mode,world", CASES, ids=[f"{m}-w{w}" for m, w in CASES])
def test_tensor_parallel_matches_oracle(mode, world):
    if _ngpus() < world:
        pytest.skip(f"needs {world} GPUs")
    p = run_worker(mode, world)
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith(f"[{mode}/")]
    print("\n".join(lines))
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    assert len(lines) == world and all("ok=True" in ln for ln in lines), lines
