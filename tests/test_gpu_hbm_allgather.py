"""Softmax and vector add with the output all-gather fused into the kernel
(piton_b200_softmax_allgather_f32, piton_b200_add_allgather_f32), on one GPU: every "rank's"
full output is a buffer of this device, so the kernel's stores land in local memory and all of
them can be read back.  This rank's rows / elements must appear, bit for bit the same as the
single-device launch, in every rank's output at its offset, and nothing else may be touched.
The same kernels over NVLink on two GPUs run in test_gpu_multi.py."""

import pytest

from piton_b200 import sharding
from piton_b200.kernels import add_kernel, softmax_kernel

pytestmark = pytest.mark.gpu
SENTINEL = -1234.5


@pytest.mark.parametrize("world,rank,rows,n", [(2, 0, 37, 781 + 3), (2, 1, 64, 1024), (4, 3, 10, 4096),
                                               (8, 6, 5, 16384), (1, 0, 9, 32768), (3, 1, 100, 256)])
def test_softmax_rows_reach_every_rank(cuda, world, rank, rows, n):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(world * 1000 + n)
    x = torch.randn(rows, n, device="cuda", generator=g) * 4
    x[:, ::97] = float("-inf")
    x[:, 1] = 0.0                                            # never a whole row of -inf
    ld = n + 8
    outs = [torch.full((world * rows, ld), SENTINEL, device="cuda") for _ in range(world)]
    r0 = rank * rows
    sharding.softmax_allgather(x, [o.data_ptr() for o in outs], rank, r0, ld)
    plain = torch.empty_like(x)
    softmax_kernel[(rows,)](plain, x, n, n, n, BLOCK_SIZE=1 << (n - 1).bit_length(), device="b200")
    torch.cuda.synchronize()
    for r, o in enumerate(outs):
        assert torch.equal(o[r0:r0 + rows, :n], plain), r          # the same bits as the plain launch
        assert bool((o[r0:r0 + rows, n:] == SENTINEL).all()), r
        assert bool((o[:r0] == SENTINEL).all()) and bool((o[r0 + rows:] == SENTINEL).all()), r
    ref = torch.softmax(x.double(), 1)
    assert float(((plain.double() - ref).abs() / ref.abs().clamp_min(1e-37)).max()) <= 1e-5


@pytest.mark.parametrize("world,rank,n", [(2, 1, 4096), (4, 0, 65536 + 4), (8, 7, 1 << 20), (1, 0, 1000)])
def test_add_elements_reach_every_rank(cuda, world, rank, n):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(n)
    x = torch.rand(n, device="cuda", generator=g) * 2 - 1
    y = torch.rand(n, device="cuda", generator=g) * 2 - 1
    outs = [torch.full((world * n + 4,), SENTINEL, device="cuda") for _ in range(world)]
    e0 = rank * n
    sharding.add_allgather(x, y, [o.data_ptr() for o in outs], rank, e0)
    plain = torch.empty_like(x)
    add_kernel[(-(-n // 1024),)](x, y, plain, n, BLOCK_SIZE=1024, device="b200")
    torch.cuda.synchronize()
    assert torch.equal(plain, x + y)
    for r, o in enumerate(outs):
        assert torch.equal(o[e0:e0 + n], plain), r
        assert bool((o[:e0] == SENTINEL).all()) and bool((o[e0 + n:] == SENTINEL).all()), r


def test_fused_allgather_argument_checks(cuda):
    torch = cuda
    x = torch.zeros(4, 10, device="cuda")                     # n % 4 != 0
    out = torch.zeros(8, 12, device="cuda")
    with pytest.raises(ValueError):
        sharding.softmax_allgather(x, [out.data_ptr()] * 2, 0, 0, 12)
    v = torch.zeros(6, device="cuda")                         # n % 4 != 0
    with pytest.raises(ValueError):
        sharding.add_allgather(v, v, [out.data_ptr()], 0, 0)
    w = torch.zeros(8, device="cuda")
    with pytest.raises(ValueError):
        sharding.add_allgather(w, w, [out.data_ptr(), 0], 0, 0)  # a NULL peer
