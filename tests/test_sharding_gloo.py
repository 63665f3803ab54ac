"""The multi-GPU host logic on CPU: two gloo ranks shard a matmul by M rows,
a softmax by rows and a vector add by elements, all-gather the pieces and
must reproduce the single-process result; timings reduce with max over ranks.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from piton_b200 import sharding


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        M, N, K = 37, 24, 16
        a = torch.from_numpy(rng.uniform(-1, 1, (M, K)).astype(np.float32))
        b = torch.from_numpy(rng.uniform(-1, 1, (K, N)).astype(np.float32))
        r0, per = sharding.shard(M, world, rank)
        a_pad = torch.zeros(per * world, K)
        a_pad[:M] = a
        piece = a_pad[r0:r0 + per] @ b
        c = torch.empty(per * world, N)
        sharding.gather(dist, c, piece)
        ok_mm = torch.allclose(c[:M], a @ b, atol=1e-6)

        x = torch.from_numpy(rng.standard_normal((64, 10)).astype(np.float32))
        r0, per = sharding.shard(64, world, rank)
        y = torch.empty(per * world, 10)
        sharding.gather(dist, y, torch.softmax(x[r0:r0 + per], 1))
        ok_sm = torch.allclose(y, torch.softmax(x, 1))

        n = 1000
        u, v = torch.arange(n, dtype=torch.float32), torch.ones(n)
        s0, per = sharding.shard(n, world, rank, multiple=4)
        up = torch.zeros(per * world)
        up[:n] = u
        vp = torch.zeros(per * world)
        vp[:n] = v
        out = torch.empty(per * world)
        sharding.gather(dist, out, up[s0:s0 + per] + vp[s0:s0 + per])
        ok_add = torch.equal(out[:n], u + v)

        t = sharding.max_over_ranks(dist, float(rank + 1))
        results[rank] = (ok_mm, ok_sm, ok_add, t)
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_shards_and_gathers():
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    assert len(res) == world
    for rank, (ok_mm, ok_sm, ok_add, t) in res.items():
        assert ok_mm and ok_sm and ok_add, rank
        assert t == float(world)


def test_shard_arithmetic():
    assert sharding.shard(8192, 8, 3) == (3072, 1024)
    assert sharding.shard(1797, 8, 7) == (7 * 225, 225)
    assert sharding.shard(10, 4, 0, multiple=4) == (0, 4)
    with pytest.raises(ZeroDivisionError):
        sharding.shard(10, 0, 0)


def _attention(q, k, v):
    s = (q @ k.transpose(1, 2)) / q.shape[-1] ** 0.5
    n = q.shape[1]
    s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
    return torch.softmax(s, -1) @ v


def _attention_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(3)
        heads, n, d = 6, 32, 16                      # batch x head flattened, as the bench shards it
        q, k, v = (torch.randn(heads, n, d, generator=g) for _ in range(3))
        h0, per = sharding.shard(heads, world, rank)
        out = torch.empty(per * world, n, d)
        sharding.gather(dist, out, _attention(q[h0:h0 + per], k[h0:h0 + per], v[h0:h0 + per]))
        results[rank] = bool(torch.allclose(out[:heads], _attention(q, k, v), atol=1e-6))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_attention_by_heads():
    """Attention sharded by batch x head: each rank's heads, gathered, equal the whole."""
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_attention_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    assert res == {0: True, 1: True}


def test_attention_allgather_rejects_mismatched_shards():
    """The fused all-gather wrapper checks q, k, v before any library call."""
    q = torch.zeros(2, 64, 64)
    with pytest.raises(ValueError):
        sharding.attention_allgather(q, torch.zeros(3, 64, 64), q, [0, 0], 0, 0)
    with pytest.raises(ValueError):
        sharding.attention_allgather(q, q.transpose(1, 2), q, [0, 0], 0, 0)
