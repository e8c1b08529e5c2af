"""Multi-rank host logic on CPU: two gloo ranks, no GPU."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kquant_b200 import sharding


def test_shard_experts_covers_every_expert_once():
    for world in (1, 2, 4, 8):
        got = [sharding.shard_experts([1.0] * 384, world, r) for r in range(world)]
        assert sorted(e for s in got for e in s) == list(range(384))
        assert all(len(s) == 384 // world for s in got)
    costs = [3.0] * 10 + [1.0] * 30
    parts = [sharding.shard_experts(costs, 4, r) for r in range(4)]
    assert sorted(e for p in parts for e in p) == list(range(40))
    loads = [sum(costs[e] for e in p) for p in parts]
    assert max(loads) - min(loads) <= 3.0
    with pytest.raises(ValueError):
        sharding.shard_experts([1.0, 0.0], 2, 0)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # tensors 0..3; rank r owns tensors r and r+2
        num = torch.zeros(4, dtype=torch.float64)
        den = torch.zeros(4, dtype=torch.float64)
        for t in (rank, rank + 2):
            num[t] = 0.01 * (t + 1)
            den[t] = 2.0
        proxy = sharding.reduce_proxy_stats(num, den)
        scales = torch.arange(8, dtype=torch.float32).reshape(8, 1) if rank == 1 else None
        got = sharding.broadcast_shared_input_scales(("layer", "w1"), scales, 1, (8, 1), "cpu")
        from kquant_b200.exl3_encoder_backend import _SHARED_INPUT_SCALES
        q.put((rank, proxy.tolist(), got.flatten().tolist(), _SHARED_INPUT_SCALES[("layer", "w1")] is got))
    finally:
        dist.destroy_process_group()


def test_two_rank_proxy_reduce_and_scale_broadcast():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, proxy, scales, registered in out:
        assert proxy == pytest.approx([0.005, 0.01, 0.015, 0.02])
        assert scales == list(map(float, range(8)))
        assert registered
