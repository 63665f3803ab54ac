"""Launches on page-locked numpy arrays large enough for the chunked host-buffer path
(runtime/cuda ``_pipelined_on_host``): the copies in and back of add, softmax and attention overlap
the launches chunk by chunk.  Each result must equal, bit for bit, the same launch on CUDA tensors
(the same kernels on the same data, only split into chunks of whole programs / rows / heads), and
output elements the launch does not cover keep their host values, as on the generic path."""

import numpy as np
import pytest

import piton_b200 as triton
from piton_b200.kernels import add_kernel, attn_fwd_kernel, softmax_kernel
from piton_b200.runtime.cuda import pinned_empty

pytestmark = pytest.mark.gpu


def test_add_pipelined_matches_device_launch(cuda):
    torch = cuda
    n, blk = 6 * (1 << 20) + 5, 1024
    grid = (n - 3000) // blk                       # the last ~3000 elements are not covered
    rng = np.random.default_rng(11)
    x, y, out = pinned_empty((n,)), pinned_empty((n,)), pinned_empty((n,))
    x[:] = rng.uniform(-1, 1, n)
    y[:] = rng.uniform(-1, 1, n)
    out[:] = 7.0
    st = add_kernel[(grid,)](x, y, out, n, BLOCK_SIZE=blk, device="b200").last_stats
    assert st["path"] == "add_vec4_host_pipelined" and st["launches"] > 1
    dx, dy = torch.from_numpy(x).cuda(), torch.from_numpy(y).cuda()
    dout = torch.full((n,), 7.0, device="cuda")
    add_kernel[(grid,)](dx, dy, dout, n, BLOCK_SIZE=blk, device="b200")
    np.testing.assert_array_equal(out.view(np.uint32), dout.cpu().numpy().view(np.uint32))
    assert np.all(out[grid * blk:] == 7.0)


def test_softmax_pipelined_matches_device_launch(cuda):
    torch = cuda
    rows, cols = 4096, 4096
    rng = np.random.default_rng(12)
    x, y = pinned_empty((rows, cols)), pinned_empty((rows, cols))
    x[:] = rng.standard_normal((rows, cols)) * 4
    x[rng.random((rows, cols)) < 0.01] = -np.inf
    x[:, 0] = 1.0
    st = softmax_kernel[(rows,)](y, x, cols, cols, cols, BLOCK_SIZE=cols, device="b200").last_stats
    assert st["path"] == "softmax_host_pipelined" and st["launches"] > 1
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty_like(dx)
    softmax_kernel[(rows,)](dy, dx, cols, cols, cols, BLOCK_SIZE=cols, device="b200")
    np.testing.assert_array_equal(y.view(np.uint32), dy.cpu().numpy().view(np.uint32))


def test_attention_pipelined_matches_device_launch(cuda):
    torch = cuda
    heads, n_ctx, d = 64, 1024, 64
    g = torch.Generator(device="cuda").manual_seed(13)
    q, k, v = (torch.randn(heads, n_ctx, d, device="cuda", generator=g) for _ in range(3))
    hq, hk, hv, ho = (pinned_empty((heads, n_ctx, d)) for _ in range(4))
    for h_, t_ in ((hq, q), (hk, k), (hv, v)):
        torch.from_numpy(h_).copy_(t_)
    sd, sm = n_ctx * d, float(1.0 / np.sqrt(d))
    launch = attn_fwd_kernel[(triton.cdiv(n_ctx, 64), heads)]
    args = (sm, sd, d, sd, d, 1, sd, d, sd, d, n_ctx)
    consts = dict(HEAD_DIM=d, BLOCK_M=64, BLOCK_N=64, CAUSAL=True, EVEN_N=True, device="b200")
    st = launch(hq, hk, hv, ho, *args, **consts).last_stats
    assert st["path"] == "attention_host_pipelined" and st["launches"] > 1
    o = torch.empty_like(q)
    launch(q, k, v, o, *args, **consts)
    np.testing.assert_array_equal(ho.view(np.uint32), o.cpu().numpy().view(np.uint32))


def test_pageable_or_small_arrays_take_the_generic_path(cuda):
    rows, cols = 4096, 4096
    x = np.random.default_rng(14).standard_normal((rows, cols)).astype(np.float32)   # not page-locked
    y = np.empty_like(x)
    st = softmax_kernel[(rows,)](y, x, cols, cols, cols, BLOCK_SIZE=cols, device="b200").last_stats
    assert st["path"] == "softmax"
    xs, ys = pinned_empty((64, 256)), pinned_empty((64, 256))                          # under the size threshold
    xs[:] = 1.0
    st = softmax_kernel[(64,)](ys, xs, 256, 256, 256, BLOCK_SIZE=256, device="b200").last_stats
    assert st["path"] == "softmax"
    np.testing.assert_allclose(ys, 1.0 / 256, rtol=1e-6)
