"""Multi-GPU matmul with the all-gather fused into the GEMM epilogue (NVLink peer
stores, or multimem stores to an NVSwitch multicast address), on 2 GPUs when
the box has them (skipped otherwise).  Every rank must
end with the full C = A @ B: rows computed by every rank are checked against
float64 on every rank."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results, kind="peer"):
    import datetime

    import torch.distributed as dist

    from piton_b200 import sharding
    from piton_b200.runtime.cuda import _lib
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    out = None
    try:
        M, N, K = 1024, 768, 640
        g = torch.Generator(device="cuda").manual_seed(5)
        A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1      # same on every rank (same seed)
        B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
        r0, per = sharding.shard(M, world, rank)
        if kind == "multicast":
            out = sharding.SymmetricOutput(dist, M * N * 4)
            assert out.multicast_ptr != 0
        else:
            out = sharding.PeerOutput(dist, M * N * 4)
        for _ in range(2):
            sharding.matmul_allgather(A[r0:r0 + per], B, out, r0, N)
            torch.cuda.synchronize()
            dist.barrier()
        full = out.read(0, M * N * 4).view(np.float32).reshape(M, N)
        ref = (A.double() @ B.double()).cpu().numpy()
        err = float(np.abs(full - ref).max() / np.abs(ref).max())
        import ctypes as C
        st = C.c_int(-1)
        _lib.lib().piton_b200_device_status(C.byref(st))
        results[rank] = (err, st.value)
        dist.barrier()
    finally:
        if out is not None:
            out.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["peer", "multicast"])
def test_fused_allgather_matmul_two_gpus(kind):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if kind == "multicast":
        from piton_b200.sharding import SymmetricOutput
        if not SymmetricOutput.multicast_supported(0):
            pytest.skip("no NVSwitch multicast on this box")
    import torch.multiprocessing as mp
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_worker, args=(2, _port(), results, kind), nprocs=2, join=True)
        res = dict(results)
    assert len(res) == 2
    for rank, (err, status) in res.items():
        assert status == 0, rank
        assert err <= 4e-6, (rank, err)


def _allgather_worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    from piton_b200 import sharding
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    out = None
    try:
        ok = True
        for n in (4096, 1001):                       # 16-byte pieces, and byte stores
            out = sharding.PeerOutput(dist, world * n * 4)
            piece = torch.arange(n, device="cuda", dtype=torch.float32) + 1000.0 * (rank + 1)
            sharding.allgather_pieces(piece, out)
            torch.cuda.synchronize()
            dist.barrier()
            full = out.read(0, world * n * 4).view(np.float32).reshape(world, n)
            want = np.arange(n, dtype=np.float32)[None, :] + 1000.0 * (np.arange(world, dtype=np.float32)[:, None] + 1)
            ok = ok and bool(np.array_equal(full, want))
            dist.barrier()
            out.close()
            out = None
        results[rank] = ok
        dist.barrier()
    finally:
        if out is not None:
            out.close()
        dist.destroy_process_group()


def test_library_allgather_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_allgather_worker, args=(2, _port(), results), nprocs=2, join=True)
        res = dict(results)
    assert res == {0: True, 1: True}


def _host_sharded_worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    from piton_b200 import sharding
    from piton_b200.runtime.cuda import pinned_empty
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    hs = None
    try:
        M, N, K = 2048, 768, 512
        rng = np.random.default_rng(3)
        a_full = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
        r0, per = sharding.shard(M, world, rank)
        A, B, Cm = pinned_empty((per, K)), pinned_empty((K, N)), pinned_empty((per, N))
        A[...], B[...] = a_full[r0:r0 + per], b
        hs = sharding.HostShardedMatmul(dist, per, N, K)
        errs = []
        for _ in range(2):
            Cm[...] = np.nan
            hs(A, B, Cm)
            ref = a_full[r0:r0 + per].astype(np.float64) @ b.astype(np.float64)
            errs.append(float(np.abs(Cm - ref).max() / np.abs(ref).max()))
        results[rank] = max(errs)
        dist.barrier()
    finally:
        if hs is not None:
            hs.close()
        dist.destroy_process_group()


def test_host_sharded_matmul_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_host_sharded_worker, args=(2, _port(), results), nprocs=2, join=True)
        res = dict(results)
    assert len(res) == 2 and all(e <= 4e-6 for e in res.values()), res


def _attention_worker(rank, world, port, results):
    import datetime

    import torch.distributed as dist

    from oracle import oracle as O
    from piton_b200 import sharding
    from piton_b200.runtime.cuda import _lib
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    out = None
    try:
        heads, n = 3, 320                              # per rank; the same seed on every rank
        g = torch.Generator(device="cuda").manual_seed(11)
        q, k, v = (torch.randn(world * heads, n, 64, device="cuda", generator=g) for _ in range(3))
        h0 = rank * heads
        out = sharding.PeerOutput(dist, world * heads * n * 64 * 4)
        for _ in range(2):
            sharding.attention_allgather(q[h0:h0 + heads].contiguous(), k[h0:h0 + heads].contiguous(),
                                         v[h0:h0 + heads].contiguous(), out.peer_ptrs, rank, h0, causal=True)
            torch.cuda.synchronize()
            dist.barrier()
        full = out.read(0, world * heads * n * 64 * 4).view(np.float32).reshape(world * heads, n, 64)
        ref = O.attention_f64(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy(), True)
        import ctypes as C
        st = C.c_int(-1)
        _lib.lib().piton_b200_device_status(C.byref(st))
        results[rank] = (float(np.abs(full - ref).max()), st.value)
        dist.barrier()
    finally:
        if out is not None:
            out.close()
        dist.destroy_process_group()


def test_fused_allgather_attention_two_gpus():
    """Every rank ends with all heads: its own stored by the softmax warps, the other rank's by
    that rank's gather warp over NVLink."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_attention_worker, args=(2, _port(), results), nprocs=2, join=True)
        res = dict(results)
    assert len(res) == 2
    for rank, (err, status) in res.items():
        assert status == 0, rank
        assert err <= 2e-5, (rank, err)


def _hbm_worker(rank, world, port, results):
    """Softmax by rows and add by elements, each rank storing its piece into every rank's full
    output from inside the kernel (NVLink peer stores); every rank must end with the whole."""
    import datetime

    import torch.distributed as dist

    from piton_b200 import sharding
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    outs = []
    try:
        rows, n = 256, 4096
        g = torch.Generator(device="cuda").manual_seed(9)
        x = torch.randn(rows, n, device="cuda", generator=g) * 4      # same on every rank (same seed)
        r0, per = sharding.shard(rows, world, rank)
        sm = sharding.PeerOutput(dist, rows * n * 4)
        outs.append(sm)
        ne = 1 << 20
        u = torch.rand(ne, device="cuda", generator=g) * 2 - 1
        v = torch.rand(ne, device="cuda", generator=g) * 2 - 1
        e0, eper = sharding.shard(ne, world, rank, multiple=4)
        ad = sharding.PeerOutput(dist, ne * 4)
        outs.append(ad)
        for _ in range(2):
            sharding.softmax_allgather(x[r0:r0 + per], sm.peer_ptrs, rank, r0, n)
            sharding.add_allgather(u[e0:e0 + eper], v[e0:e0 + eper], ad.peer_ptrs, rank, e0)
            torch.cuda.synchronize()
            dist.barrier()
        got_sm = sm.read(0, rows * n * 4).view(np.float32).reshape(rows, n)
        ref = torch.softmax(x.double(), 1).cpu().numpy()
        err_sm = float((np.abs(got_sm - ref) / np.maximum(np.abs(ref), 1e-37)).max())
        got_add = ad.read(0, ne * 4).view(np.float32)
        exact_add = bool(np.array_equal(got_add, (u + v).cpu().numpy()))
        results[rank] = (err_sm, exact_add)
        dist.barrier()
    finally:
        for o in outs:
            o.close()
        dist.destroy_process_group()


def test_fused_allgather_softmax_and_add_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_hbm_worker, args=(2, _port(), results), nprocs=2, join=True)
        res = dict(results)
    assert len(res) == 2
    for rank, (err_sm, exact_add) in res.items():
        assert err_sm <= 1e-5, (rank, err_sm)
        assert exact_add, rank
