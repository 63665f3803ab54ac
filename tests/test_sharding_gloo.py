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


def _batch_worker(rank, world, port, results):
    """Each rank classifies / decodes only its piece of the batch with the oracle's host models
    and the gathered result must be the single-process one, row for row."""
    from oracle import oracle as O
    from oracle import tinygpt_ref
    from piton_b200 import tinygpt, workloads as W
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        images, model = W.digits_images(1797, 0), W.digits_model(0)
        pred = sharding.run_batch_sharded(
            dist, lambda piece: torch.from_numpy(np.argmax(O.qpu_mlp(piece, model)[:, :10], 1)), images)
        w = tinygpt.init_weights(0)
        prompts = tinygpt.random_prompts(256, seed=100)
        toks = sharding.run_batch_sharded(
            dist, lambda piece: torch.from_numpy(tinygpt_ref.generate(w, piece, tinygpt.NEW_TOKENS)[0]), prompts)
        results[rank] = (pred.numpy().tolist(), toks.numpy().tolist())
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_batch_sharding_of_mlp_and_tinygpt():
    """The digits predict (1797 images, the last rank's piece padded with zero images) and a
    256-sequence TinyGPT greedy decode, sharded by batch over two gloo ranks: the gathered
    argmax and tokens equal the single-process result exactly, on both ranks."""
    from oracle import oracle as O
    from oracle import tinygpt_ref
    from piton_b200 import tinygpt, workloads as W
    images, model = W.digits_images(1797, 0), W.digits_model(0)
    want_pred = np.argmax(O.qpu_mlp(images, model)[:, :10], 1)
    w = tinygpt.init_weights(0)
    want_toks = tinygpt_ref.generate(w, tinygpt.random_prompts(256, seed=100), tinygpt.NEW_TOKENS)[0]
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_batch_worker, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    assert sorted(res) == [0, 1]
    for rank, (pred, toks) in res.items():
        np.testing.assert_array_equal(np.array(pred), want_pred, err_msg=f"rank {rank}")
        np.testing.assert_array_equal(np.array(toks), want_toks, err_msg=f"rank {rank}")


def test_batch_piece_pads_the_last_rank():
    batch = np.arange(10 * 3).reshape(10, 3)
    p0, s0 = sharding.batch_piece(batch, 4, 0)
    p3, s3 = sharding.batch_piece(batch, 4, 3)
    assert (s0, s3) == (0, 9) and p0.shape == p3.shape == (3, 3)
    np.testing.assert_array_equal(p3[0], batch[9])
    assert not p3[1:].any()
    one, _ = sharding.batch_piece(batch, 1, 0)
    np.testing.assert_array_equal(one, batch)
