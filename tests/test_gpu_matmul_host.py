"""The host-buffer matmul (piton_b200_matmul_f32_host): numpy launches whose
copies are pipelined with the GEMM in row blocks give the same bits as the same
launch on device tensors, for one block, several blocks, a ragged tail that
joins the block before it, K not a multiple of 4, pinned and pageable arrays."""

import ctypes as C

import numpy as np
import pytest

import piton_b200 as triton
from piton_b200.kernels import matmul_kernel
from piton_b200.runtime.cuda import _lib, lib, pinned_empty

pytestmark = pytest.mark.gpu


def run(a, b, c, M, N, K):
    grid = (triton.cdiv(M, 8) * triton.cdiv(N, 64),)
    return matmul_kernel[grid](a, b, c, M, N, K, K, 1, N, 1, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64,
                               BLOCK_SIZE_K=8, GROUP_SIZE_M=8, device="b200").last_stats


@pytest.mark.parametrize("M,N,K,pinned", [(1024, 1024, 1024, True), (2200, 384, 256, True), (2100, 640, 300, False),
                                          (4096, 512, 96, True), (300, 200, 1000, False)])
def test_host_path_same_bits_as_device_path(cuda, M, N, K, pinned):
    torch = cuda
    rng = np.random.default_rng(M + N + K)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    if pinned:
        pa, pb = pinned_empty((M, K)), pinned_empty((K, N))
        pa[...], pb[...] = a, b
        a, b = pa, pb
        c = pinned_empty((M, N))
    else:
        c = np.empty((M, N), np.float32)
    c[...] = np.nan
    st = run(a, b, c, M, N, K)
    assert st["path"] == "tcgen05_f16x3_host_pipelined"
    assert st["h2d_bytes"] == 4 * (M * K + K * N) and st["d2h_bytes"] == 4 * M * N
    ta, tb = torch.from_numpy(np.array(a)).cuda(), torch.from_numpy(np.array(b)).cuda()
    tc = torch.full((M, N), float("nan"), device="cuda")
    st2 = run(ta, tb, tc, M, N, K)
    assert st2["path"] == "tcgen05_f16x3"
    np.testing.assert_array_equal(c.view(np.uint32), tc.cpu().numpy().view(np.uint32))
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert np.abs(c - ref).max() / np.abs(ref).max() <= max(4e-6, 1e-7 * np.sqrt(K))


def test_repeated_calls_and_other_shapes_between(cuda):
    """The copy streams and events are reused: back-to-back calls, with a call of another
    shape between them, keep giving the same answer."""
    rng = np.random.default_rng(7)
    M, N, K = 2304, 512, 512
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    first = np.zeros((M, N), np.float32)
    run(a, b, first, M, N, K)
    a2 = rng.uniform(-1, 1, (1500, 700)).astype(np.float32)
    b2 = rng.uniform(-1, 1, (700, 300)).astype(np.float32)
    c2 = np.zeros((1500, 300), np.float32)
    run(a2, b2, c2, 1500, 300, 700)
    for _ in range(3):
        again = np.zeros((M, N), np.float32)
        run(a, b, again, M, N, K)
        np.testing.assert_array_equal(again.view(np.uint32), first.view(np.uint32))
    ref = a2.astype(np.float64) @ b2.astype(np.float64)
    assert np.abs(c2 - ref).max() / np.abs(ref).max() <= 4e-6


def test_strided_or_aliased_launches_take_the_generic_path(cuda):
    rng = np.random.default_rng(3)
    M = N = K = 512
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    bt = np.ascontiguousarray(rng.uniform(-1, 1, (K, N)).astype(np.float32).T)   # B through (1, K) strides
    c = np.zeros((M, N), np.float32)
    grid = (triton.cdiv(M, 8) * triton.cdiv(N, 64),)
    st = matmul_kernel[grid](a, bt, c, M, N, K, K, 1, 1, K, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8,
                             GROUP_SIZE_M=8, device="b200").last_stats
    assert st["path"] == "tcgen05_f16x3"
    ref = a.astype(np.float64) @ bt.T.astype(np.float64)
    assert np.abs(c - ref).max() / np.abs(ref).max() <= 4e-6
    # C is A (in-place square product): the generic path, which copies each array in first
    x = rng.uniform(-1, 1, (M, M)).astype(np.float32)
    y = rng.uniform(-1, 1, (M, M)).astype(np.float32)
    want = x.astype(np.float64) @ y.astype(np.float64)
    st = run(x, y, x, M, M, M)
    assert st["path"] == "tcgen05_f16x3"
    assert np.abs(x - want).max() / np.abs(want).max() <= 4e-6


def test_c_abi_rejects_overlap_and_unsupported_layouts(cuda):
    M = N = K = 1024
    a = np.zeros((M, K), np.float32)
    b = np.zeros((K, N), np.float32)
    args = _lib.MatmulArgs(a.ctypes.data, b.ctypes.data, a.ctypes.data, M, N, K, K, 1, N, 1, N, 1, 8, 64, 8, 8,
                           (M // 8) * (N // 64), 0, 0, 0, 0)
    ws = lib().piton_b200_matmul_host_workspace_size(C.byref(args))
    assert ws > 0
    import torch
    buf = torch.empty(ws, dtype=torch.uint8, device="cuda")
    args.workspace, args.workspace_bytes = buf.data_ptr(), ws
    assert lib().piton_b200_matmul_f32_host(C.byref(args), None) == _lib.EINVAL
    assert b"overlaps" in lib().piton_b200_last_error()
    args.stride_bn, args.stride_bk = K, 1
    assert lib().piton_b200_matmul_host_workspace_size(C.byref(args)) == 0
    assert lib().piton_b200_matmul_f32_host(C.byref(args), None) == _lib.ENOTSUP
    args.stride_bn, args.stride_bk = 1, N
    args.workspace_bytes = ws - 1
    c = np.zeros((M, N), np.float32)
    args.c = c.ctypes.data
    assert lib().piton_b200_matmul_f32_host(C.byref(args), None) == _lib.EWORKSPACE
    torch.cuda.synchronize()


@pytest.mark.parametrize("where", ["hdh", "dhh", "hhd", "ddd"])
def test_mixed_host_and_device_operands(cuda, where):
    """Operands already in device memory are used in place (A, B, C = host or device in the
    order of `where`); every mix gives the bits of the device-buffer call."""
    torch = cuda
    M, N, K = 2304, 640, 384
    rng = np.random.default_rng(17)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    want = torch.empty(M, N, device="cuda")
    run(ta, tb, want, M, N, K)
    ha, hb, hc = pinned_empty((M, K)), pinned_empty((K, N)), pinned_empty((M, N))
    ha[...], hb[...], hc[...] = a, b, np.nan
    dc = torch.full((M, N), float("nan"), device="cuda")
    ptr = {"a": (ha.ctypes.data, ta.data_ptr()), "b": (hb.ctypes.data, tb.data_ptr()),
           "c": (hc.ctypes.data, dc.data_ptr())}
    pa, pb, pc = (ptr[k][where[i] == "d"] for i, k in enumerate("abc"))
    args = _lib.MatmulArgs(pa, pb, pc, M, N, K, K, 1, N, 1, N, 1, 8, 64, 8, 8, (M // 8) * (N // 64), 0, 0, 0, 0)
    ws = lib().piton_b200_matmul_host_workspace_size(C.byref(args))
    assert ws > 0
    buf = torch.empty(ws, dtype=torch.uint8, device="cuda")
    args.workspace, args.workspace_bytes = buf.data_ptr(), ws
    _lib.check(lib().piton_b200_matmul_f32_host(C.byref(args), None), "matmul host")
    torch.cuda.synchronize()
    got = dc.cpu().numpy() if where[2] == "d" else hc
    np.testing.assert_array_equal(got.view(np.uint32), want.cpu().numpy().view(np.uint32))
