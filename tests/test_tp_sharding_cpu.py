"""Tensor-parallel sharding scheme on CPU (world_size 2, gloo): each rank
computes the decoder layer for its shard with the oracle's math, exactly the
columns/rows libmb200 packs for that rank (mb_decoder_layer_create):

  * q heads [r*Hq/P, (r+1)*Hq/P), kv heads [r*Hkv/P, ...) of W_qkv's columns;
  * W_o rows of this rank's q features (row-sharded), summed by all-reduce,
    residual added on rank 0 only;
  * gate/up features [r*FF/P, ...) of W_gu, W_down rows of the same features,
    summed by all-reduce, residual on rank 0 only.

The all-reduced output must equal the unsharded layer. No GPU is involved.
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle.ops as O

D, H, HKV, FF, DH, S, BASE, EPS = 256, 4, 2, 256, 64, 12, 10000.0, 1e-5


def _weights():
    rng = np.random.default_rng(21)
    r = lambda *s: rng.standard_normal(s) * 0.1
    return rng.standard_normal((1, S, D)), [r(D, D + 2 * HKV * DH), r(D, D), r(D, 2 * FF),
                                            r(FF, D)]


def _shard_forward(rank, world, x, W):
    Wqkv, Wo, Wgu, Wd = W
    hq, hkv, ff = H // world, HKV // world, FF // world
    q_cols = np.arange(rank * hq * DH, (rank + 1) * hq * DH)
    k_cols = D + np.arange(rank * hkv * DH, (rank + 1) * hkv * DH)
    v_cols = D + HKV * DH + np.arange(rank * hkv * DH, (rank + 1) * hkv * DH)
    pos = np.arange(S)
    h = O.rms_norm(x, EPS)
    q = (h @ Wqkv[:, q_cols]).reshape(1, S, hq, DH).transpose(0, 2, 1, 3)
    k = (h @ Wqkv[:, k_cols]).reshape(1, S, hkv, DH).transpose(0, 2, 1, 3)
    v = (h @ Wqkv[:, v_cols]).reshape(1, S, hkv, DH).transpose(0, 2, 1, 3)
    q, k = O.rope(q, pos, BASE), O.rope(k, pos, BASE)
    G = H // HKV
    kr, vr = np.repeat(k, G, axis=1), np.repeat(v, G, axis=1)
    sc = q @ kr.transpose(0, 1, 3, 2) / np.sqrt(DH)
    sc = np.where(pos[None, :] > pos[:, None], -np.inf, sc)
    p = np.exp(sc - sc.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    a = (p @ vr).transpose(0, 2, 1, 3).reshape(1, S, hq * DH)
    part = a @ Wo[q_cols]
    if rank == 0:
        part = part + x
    t = torch.from_numpy(np.ascontiguousarray(part))
    dist.all_reduce(t)
    x1 = t.numpy()
    h2 = O.rms_norm(x1, EPS)
    f = np.arange(rank * ff, (rank + 1) * ff)
    g, u = h2 @ Wgu[:, f], h2 @ Wgu[:, FF + f]
    part2 = (O.silu(g) * u) @ Wd[f]
    if rank == 0:
        part2 = part2 + x1
    t2 = torch.from_numpy(np.ascontiguousarray(part2))
    dist.all_reduce(t2)
    return t2.numpy()


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x, W = _weights()
    y = _shard_forward(rank, world, x, W)
    if rank == 0:
        q.put(y)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_shards_sum_to_full_layer(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29611
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    y = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    x, W = _weights()
    ref = O.decoder_layer(x, *W, H=H, H_kv=HKV, base=BASE, eps=EPS, causal=True, acc=np.float64)
    np.testing.assert_allclose(y, ref, rtol=1e-6, atol=1e-6)  # oracle returns float32


def test_rank_that_never_joins_times_out():
    """A rank that never joins: the other side's rendezvous fails with a timeout
    error on the host instead of hanging (fault made on the host, no GPU)."""
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT="29623")
    with pytest.raises(Exception):
        dist.init_process_group("gloo", rank=0, world_size=2,
                                timeout=datetime.timedelta(seconds=3))
    if dist.is_initialized():
        dist.destroy_process_group()
