"""The attention with the output all-gather fused into the kernel
(piton_b200_attention_allgather_f32), on one GPU: every "rank's" full output is a buffer of
this device, so the gather warp's stores land in local memory and all of them can be read
back.  This rank's heads must appear, bit for bit the same, in every rank's output at its head
offset, within ATOL of float64, and nothing else may be touched.  The same kernel on two GPUs
(NVLink peer stores) runs in test_gpu_multi.py."""

import numpy as np
import pytest

from oracle import oracle as O
from piton_b200 import sharding
from piton_b200.kernels import attn_fwd_kernel

pytestmark = pytest.mark.gpu
ATOL = 2e-5
SENTINEL = -1234.5


def _status():
    import ctypes
    from piton_b200.runtime.cuda._lib import lib
    st = ctypes.c_int(-1)
    assert lib().piton_b200_device_status(ctypes.byref(st)) == 0
    return st.value


@pytest.mark.parametrize("world,rank,heads,n,causal", [(2, 0, 3, 256, True), (2, 1, 2, 200, True),
                                                       (4, 2, 2, 513, False), (8, 5, 1, 1024, True),
                                                       (1, 0, 2, 128, True)])
def test_every_rank_output_gets_this_rank_heads(cuda, world, rank, heads, n, causal):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(world * 100 + n)
    q, k, v = (torch.randn(heads, n, 64, device="cuda", generator=g) for _ in range(3))
    h0, total = rank * heads, world * heads
    outs = [torch.full((total, n, 64), SENTINEL, device="cuda") for _ in range(world)]
    sharding.attention_allgather(q, k, v, [o.data_ptr() for o in outs], rank, h0, causal=causal)
    torch.cuda.synchronize()
    assert _status() == 0
    mine = outs[rank][h0:h0 + heads]
    for r, o in enumerate(outs):
        assert torch.equal(o[h0:h0 + heads], mine), r            # the peers hold copies of the same bits
        assert bool((o[:h0] == SENTINEL).all()) and bool((o[h0 + heads:] == SENTINEL).all()), r
    qn, kn, vn = (t.cpu().numpy() for t in (q, k, v))
    np.testing.assert_allclose(mine.cpu().numpy(), O.attention_f64(qn, kn, vn, causal), rtol=0, atol=ATOL)
    # the single-device call on the same inputs
    plain = torch.empty_like(q)
    sd = n * 64
    attn_fwd_kernel[(-(-n // 64), heads)](q, k, v, plain, 0.125, sd, 64, sd, 64, 1, sd, 64, sd, 64, n, HEAD_DIM=64,
                                          BLOCK_M=64, BLOCK_N=64, CAUSAL=causal, EVEN_N=n % 64 == 0,
                                          device="b200")
    torch.cuda.synchronize()
    assert float((plain - mine).abs().max()) <= ATOL


def test_repeated_calls_overwrite_in_place(cuda):
    """Two calls into the same outputs (as every benchmark step does): the second result replaces
    the first, and the outputs hold only the second call's values."""
    torch = cuda
    world, heads, n = 2, 2, 384
    outs = [torch.full((world * heads, n, 64), SENTINEL, device="cuda") for _ in range(world)]
    ptrs = [o.data_ptr() for o in outs]
    for seed in (1, 2):
        g = torch.Generator(device="cuda").manual_seed(seed)
        q, k, v = (torch.randn(heads, n, 64, device="cuda", generator=g) for _ in range(3))
        sharding.attention_allgather(q, k, v, ptrs, 1, heads, causal=True)
    torch.cuda.synchronize()
    assert _status() == 0
    want = O.attention_f64(*(t.cpu().numpy() for t in (q, k, v)), True)
    for o in outs:
        np.testing.assert_allclose(o[heads:].cpu().numpy(), want, rtol=0, atol=ATOL)
        assert bool((o[:heads] == SENTINEL).all())
