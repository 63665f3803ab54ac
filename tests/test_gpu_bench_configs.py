"""Parity at the benchmark's own configurations, so the headline numbers come from
shapes that a failing test guards.

* matmul 8192^3 through ``kernel[grid]`` (the CTA-pair tcgen05 kernel, K = 8192 in
  chunked TMEM accumulation): 64 rows of C, two in every 256-row pair tile (one in
  each CTA's half, first and last row included), against the oracle's restatement
  of the emulator (<= 2e-5 * sqrt(K) normalised, the hot-path tolerance) and against
  float64 at fp32 level; every element of C through a float64 checksum C @ x
  against A @ (B @ x) for a random x.
* causal attention B=32, H=32, S=4096, D=64 through ``kernel[grid]`` (the persistent
  tcgen05 schedule): four whole heads (first, middle, last and one more: every query
  block, the diagonal and the last, heaviest block) against float64 at ATOL 2e-5;
  every head's first row (it attends to key 0 alone, so it equals V's first row)
  and, for every row of every head, the convex-combination bound
  |O[i]| <= max_{j <= i} |V[j]| that a causal softmax-weighted average obeys.
* the digits predict and the TinyGPT batch-256 decode sharded by batch over two
  gloo ranks (on this one GPU): gathered argmax and tokens equal the
  single-process result exactly.
"""

import math
import os
import socket

import numpy as np
import pytest

import piton_b200 as triton
from oracle import oracle as O
from piton_b200.kernels import attn_fwd_kernel, matmul_kernel

pytestmark = pytest.mark.gpu
ATOL = 2e-5


def fp32_bound(K):
    return max(4e-6, 1e-7 * math.sqrt(K))


def pair_tile_rows(M, tile=256):
    """Two rows per 256-row CTA-pair tile, one in each CTA's 128-row half, first and last row of C
    included."""
    rows = []
    for t in range(M // tile):
        rows.append(t * tile + (t * 37) % 128)
        rows.append(t * tile + 128 + (t * 53 + 5) % 128)
    rows[-1] = M - 1
    return np.array(sorted(set(rows)))


def test_matmul_8192_cubed(cuda):
    torch = cuda
    M = N = K = 8192
    rng = np.random.default_rng(8192)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    A, B = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    Cd = torch.full((M, N), float("nan"), device="cuda")
    st = matmul_kernel[(triton.cdiv(M, 8) * triton.cdiv(N, 64),)](
        A, B, Cd, M, N, K, K, 1, N, 1, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8,
        device="b200").last_stats
    assert st["path"] == "tcgen05_f16x3"
    rows = pair_tile_rows(M)
    assert len(rows) == 64
    c = Cd[torch.from_numpy(rows).cuda()].cpu().numpy()
    ref = O.qpu_matmul(a[rows], b, threads=os.cpu_count() or 1)
    err_oracle = float(np.abs(c - ref).max() / np.abs(ref).max())
    exact = a[rows].astype(np.float64) @ b.astype(np.float64)
    err_f64 = float(np.abs(c - exact).max() / np.abs(exact).max())
    assert err_oracle <= 2e-5 * math.sqrt(K), err_oracle
    assert err_f64 <= fp32_bound(K), err_f64
    # every element: a float64 checksum of the whole product
    assert bool(torch.isfinite(Cd).all())
    x = torch.randn(N, dtype=torch.float64, device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    got = Cd.double() @ x
    want = A.double() @ (B.double() @ x)
    err_sum = float((got - want).abs().max() / want.abs().max())
    assert err_sum <= fp32_bound(K), err_sum


def test_attention_b32_h32_s4096_d64_causal(cuda):
    torch = cuda
    BH, S, D = 32 * 32, 4096, 64
    g = torch.Generator(device="cuda").manual_seed(4096)
    q, k, v = (torch.randn(BH, S, D, device="cuda", generator=g) for _ in range(3))
    o = torch.full_like(q, float("nan"))
    sd = S * D
    st = attn_fwd_kernel[(S // 2, BH)](q, k, v, o, 1.0 / math.sqrt(D), sd, D, sd, D, 1, sd, D, sd, D, S,
                                       HEAD_DIM=D, BLOCK_M=2, BLOCK_N=16, CAUSAL=True, EVEN_N=True,
                                       device="b200").last_stats
    assert st["path"] == "tcgen05_f16x3"
    assert bool(torch.isfinite(o).all())
    for h in (0, BH // 2, 701, BH - 1):
        ref = O.attention_f64(q[h].cpu().numpy(), k[h].cpu().numpy(), v[h].cpu().numpy(), True)
        err = float(np.abs(o[h].cpu().numpy() - ref).max())
        assert err <= ATOL, (h, err)
    # every head: row 0 sees key 0 only
    err0 = float((o[:, 0] - v[:, 0]).abs().max())
    assert err0 <= ATOL, err0
    # every row of every head is a softmax-weighted average of V rows 0..i
    bound = torch.cummax(v.abs(), dim=1).values
    excess = float((o.abs() - bound).max())
    assert excess <= ATOL, excess


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch_rank(rank, world, port, results):
    """One gloo rank on cuda:0: its piece of the batch through the B200 MLP and TinyGPT decode."""
    import torch
    import torch.distributed as dist

    from piton_b200 import digits, sharding, tinygpt, workloads as W
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = digits.DigitsMLP(W.digits_model(0))

        def classify(piece):
            x = torch.from_numpy(piece).cuda()
            logits = torch.empty(len(piece), 16, device="cuda")
            pred = torch.empty(len(piece), dtype=torch.int32, device="cuda")
            model.forward_device(x, logits, pred)
            return pred.cpu()

        pred = sharding.run_batch_sharded(dist, classify, W.digits_images(1797, 0))
        gpt = tinygpt.TinyGPT(tinygpt.init_weights(0))
        toks = sharding.run_batch_sharded(dist, lambda piece: torch.from_numpy(gpt.generate(piece)),
                                          tinygpt.random_prompts(256, seed=100))
        results[rank] = (pred.numpy().tolist(), toks.numpy().tolist())
    finally:
        dist.destroy_process_group()


def test_batch_sharded_mlp_and_tinygpt_two_ranks(cuda):
    torch = cuda
    import torch.multiprocessing as mp

    from piton_b200 import digits, tinygpt, workloads as W
    images = W.digits_images(1797, 0)
    _, want_pred = digits.forward(images, W.digits_model(0), return_pred=True)
    want_toks = tinygpt.TinyGPT(tinygpt.init_weights(0)).generate(tinygpt.random_prompts(256, seed=100))
    torch.cuda.synchronize()
    world = 2
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_batch_rank, args=(world, _free_port(), results), nprocs=world, join=True)
        res = dict(results)
    assert sorted(res) == [0, 1]
    for rank, (pred, toks) in res.items():
        np.testing.assert_array_equal(np.array(pred), want_pred, err_msg=f"rank {rank}")
        np.testing.assert_array_equal(np.array(toks), want_toks, err_msg=f"rank {rank}")
