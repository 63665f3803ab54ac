"""Grouped tutorial matmul on the B200 (examples/kernels.py:18-57).

* QPU rounding mode (CUDA cores, sequential k, round-toward-zero): bit-exact
  with the oracle and the emulator goldens, negative C row stride included.
* Default mode (tcgen05 fp16 split with per-chunk scaling where the layout allows, CUDA cores else):
  normalised error max|C - C_oracle| / max|C_oracle| <= 2e-5 * sqrt(K), the
  hot-path tolerance; the float64 product is also checked at fp32 level,
  <= max(4e-6, 1e-7 * sqrt(K)) normalised -- the error of an fp32 FFMA loop is
  ~2e-6 at K = 8192, single-pass TF32 ~1e-4, tensor-core accumulation of the
  whole K without chunking ~7e-5.
"""

import math

import numpy as np
import pytest

import piton_b200 as triton
from conftest import dot_error, golden_ids, goldens
from oracle import oracle as O
from piton_b200 import workloads as W
from piton_b200.kernels import matmul_kernel
from piton_b200.runtime.launcher import Launcher, offset_ptr

pytestmark = pytest.mark.gpu
MATMUL = goldens("matmul_")
FP32_LEVEL = 1e-7      # normalised error per sqrt(K) against float64 ...
FP32_FLOOR = 4e-6      # ... and its floor for small K


def fp32_bound(K):
    return max(FP32_FLOOR, FP32_LEVEL * math.sqrt(K))


def launch(a, b, c, M, N, K, bm=8, bn=64, bk=8, g=8, grid=None, neg=False, qpu=False, c_arg=None):
    grid = grid or (triton.cdiv(M, bm) * triton.cdiv(N, bn),)
    scm = -N if neg else N
    c_arg = c_arg if c_arg is not None else (offset_ptr(c, (M - 1) * N) if neg else c)
    return Launcher(matmul_kernel, grid)(a, b, c_arg, M, N, K, K, 1, N, 1, scm, 1, BLOCK_SIZE_M=bm, BLOCK_SIZE_N=bn,
                                          BLOCK_SIZE_K=bk, GROUP_SIZE_M=g, device="b200", qpu_rounding=qpu)


@pytest.mark.parametrize("M,N,Kd", [(64, 64, 64), (72, 100, 64), (40, 70, 36), (16, 128, 32)])
def test_reference_shapes(cuda, M, N, Kd):
    rng = np.random.default_rng(42)
    a = rng.standard_normal((M, Kd)).astype(np.float32)
    b = rng.standard_normal((Kd, N)).astype(np.float32)
    c = np.full((M, N), -1.0, np.float32)
    launch(a, b, c, M, N, Kd, bk=4, g=4)
    np.testing.assert_allclose(c, a @ b, rtol=1e-4, atol=1e-4)      # tests/test_kernels.py:50


@pytest.mark.parametrize("g", MATMUL, ids=golden_ids(MATMUL))
def test_qpu_mode_bit_exact_vs_emulator(cuda, g):
    m = g.meta
    M, N, K = m["M"], m["N"], m["K"]
    a, b = W.matmul_inputs(M, N, K, m["seed"])
    store = np.zeros((M, N), np.float32)
    bm, bn, bk = m["block"]
    launch(a, b, store, M, N, K, bm, bn, bk, m["group"], neg=m["negative_stride_cm"], qpu=True)
    c = store[::-1] if m["negative_stride_cm"] else store
    ref = O.qpu_matmul(a, b, threads=8)
    np.testing.assert_array_equal(np.ascontiguousarray(c).view(np.uint32), ref.view(np.uint32))
    if "c" in g:
        np.testing.assert_array_equal(np.ascontiguousarray(c).view(np.uint32), g["c"].view(np.uint32))


@pytest.mark.parametrize("M,N,K,neg", [(128, 128, 128, False), (512, 512, 512, False), (1024, 1024, 1024, False),
                                       (1000, 777, 513, True)])
def test_config_shapes_within_dot_tolerance(cuda, M, N, K, neg):
    a, b = W.matmul_inputs(M, N, K, 0)
    store = np.zeros((M, N), np.float32)
    stats = launch(a, b, store, M, N, K, bk=4 if K % 8 else 8, neg=neg).last_stats
    c = store[::-1] if neg else store
    ref = O.qpu_matmul(a, b, threads=8)
    assert dot_error(c, ref) <= 2e-5 * math.sqrt(K), stats
    exact = a.astype(np.float64) @ b.astype(np.float64)
    assert dot_error(c, exact) <= fp32_bound(K), stats


def test_partial_grid_only_writes_its_tiles(cuda):
    M, N, K = 40, 200, 24
    a, b = W.matmul_inputs(M, N, K, 3)
    c = np.full((M, N), 9.0, np.float32)
    bm, bn, g = 8, 64, 2
    grid = 7                                   # of 5 * 4 = 20 programs
    launch(a, b, c, M, N, K, bm, bn, 8, g, grid=(grid,))
    num_pid_m, num_pid_n = 5, 4
    expect = np.full((M, N), 9.0, np.float32)
    full = a @ b
    for pid in range(grid):                    # the grouped order of examples/kernels.py:26-35
        group_id = pid // (g * num_pid_n)
        first = group_id * g
        gsize = min(num_pid_m - first, g)
        pm = first + (pid % (g * num_pid_n)) % gsize
        pn = (pid % (g * num_pid_n)) // gsize
        expect[pm * bm:(pm + 1) * bm, pn * bn:(pn + 1) * bn] = full[pm * bm:(pm + 1) * bm, pn * bn:(pn + 1) * bn]
    np.testing.assert_allclose(c, expect, rtol=1e-5, atol=1e-5)
    assert np.all(c[expect == 9.0] == 9.0)


def test_strided_and_transposed_operands(cuda):
    torch = cuda
    M, N, K = 96, 80, 72
    A = torch.randn(K, M, device="cuda").t()            # stride_am = 1, stride_ak = M
    B = torch.randn(N, K, device="cuda").t()            # stride_bk = 1, stride_bn = K
    C = torch.zeros(N, M, device="cuda").t()            # stride_cm = 1, stride_cn = M
    Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
        A, B, C, M, N, K, A.stride(0), A.stride(1), B.stride(0), B.stride(1), C.stride(0), C.stride(1),
        BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8, device="b200")
    torch.testing.assert_close(C, (A.double() @ B.double()).float(), rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("M,N,K", [(2048, 2048, 2048), (256, 384, 1000), (4096, 256, 512)])
def test_tensor_core_path_large(cuda, M, N, K):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1
    B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
    C = torch.empty(M, N, device="cuda")
    st = Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
        A, B, C, M, N, K, K, 1, N, 1, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8,
        device="b200").last_stats
    ref = A.double() @ B.double()
    err = float((C.double() - ref).abs().max() / ref.abs().max())
    assert err <= fp32_bound(K), (err, st)
    assert st["path"] == "tcgen05_f16x3"
    assert device_status() == 0


def device_status():
    import ctypes
    from piton_b200.runtime.cuda._lib import lib
    s = ctypes.c_int(-1)
    assert lib().piton_b200_device_status(ctypes.byref(s)) == 0
    return s.value


@pytest.mark.parametrize("M,N,K,neg", [(768, 520, 300, False), (1100, 300, 200, True), (512, 256, 64, False)])
def test_tensor_core_pairs_strided_c(cuda, M, N, K, neg):
    """Problems the CTA-pair kernel (2-SM MMAs, M >= 512) takes, with C transposed in
    memory (scalar stores) or with a negative row stride."""
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(M + 7 * N + K)
    A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1
    B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
    base = torch.full((N * M + 64,), 7.0, device="cuda")
    if neg:
        Cv = base[:M * N].view(M, N)
        st = Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
            A, B, offset_ptr(base, (M - 1) * N), M, N, K, K, 1, N, 1, -N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64,
            BLOCK_SIZE_K=8, GROUP_SIZE_M=8, device="b200").last_stats
        got = Cv.flip(0)
    else:
        Ct = base[:M * N].view(N, M).t()                  # stride_cm = 1, stride_cn = M
        st = Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
            A, B, Ct, M, N, K, K, 1, N, 1, Ct.stride(0), Ct.stride(1), BLOCK_SIZE_M=8, BLOCK_SIZE_N=64,
            BLOCK_SIZE_K=8, GROUP_SIZE_M=8, device="b200").last_stats
        got = Ct
    assert st["path"] == "tcgen05_f16x3"
    ref = A.double() @ B.double()
    err = float((got.double() - ref).abs().max() / ref.abs().max())
    assert err <= fp32_bound(K), err
    assert bool((base[M * N:] == 7.0).all())
    assert device_status() == 0


@pytest.mark.parametrize("M,N,K", [(1024, 8192, 256), (2048, 1000, 512), (640, 4000, 64)])
def test_tensor_core_224_wide_tiles_ragged_n(cuda, M, N, K):
    """Shapes whose tiles pack into fewer rounds 224 columns wide (the last N tile is
    partial): C's padding columns past N stay untouched."""
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(M * 3 + N)
    A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1
    B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
    ldc = N + 12
    Cp = torch.full((M, ldc), 5.0, device="cuda")
    st = Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
        A, B, Cp, M, N, K, K, 1, N, 1, ldc, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8,
        device="b200").last_stats
    assert st["path"] == "tcgen05_f16x3"
    ref = A.double() @ B.double()
    err = float((Cp[:, :N].double() - ref).abs().max() / ref.abs().max())
    assert err <= fp32_bound(K), err
    assert bool((Cp[:, N:] == 5.0).all())
    assert device_status() == 0


@pytest.mark.parametrize("K", [16, 17, 255, 256, 257, 4099])
def test_tensor_core_k_edges(cuda, K):
    # K not a multiple of the 16-wide k-block or of the 256-wide accumulation chunk
    torch = cuda
    M, N = 300, 520
    A = torch.rand(M, K, device="cuda") * 2 - 1
    B = torch.rand(K, N, device="cuda") * 2 - 1
    C = torch.full((M + 5, N), 3.0, device="cuda")
    st = Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
        A, B, C, M, N, K, K, 1, N, 1, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8,
        device="b200").last_stats
    ref = A.double() @ B.double()
    if st["path"] == "tcgen05_f16x3":
        assert device_status() == 0
    err = float((C[:M].double() - ref).abs().max() / ref.abs().max())
    assert err <= fp32_bound(K), (err, st)
    assert bool((C[M:] == 3.0).all())


@pytest.mark.parametrize("K", [16, 17, 255, 257, 1001, 4099])
def test_tensor_core_pairs_k_edges_padded_rows(cuda, K):
    """Row-major operands on the CTA-pair kernel (M >= 512) with K off the 256-wide chunk and the
    8-wide fp16 row (the split's zero tails), A's rows read from a wider padded buffer, N = 520 (a
    partial last tile), and two calls in a row on the same buffers (the workspace's earlier
    contents never reach C)."""
    torch = cuda
    M, N = 512, 520
    g = torch.Generator(device="cuda").manual_seed(K)
    lda = (K + 3) // 4 * 4 + 4                                # a multiple of 4: 16-byte rows
    A = (torch.rand(M, lda, device="cuda", generator=g) * 2 - 1)[:, :K]
    B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
    ref = A.double() @ B.double()
    for _ in range(2):
        C = torch.full((M, N), 9.0, device="cuda")
        st = Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
            A, B, C, M, N, K, A.stride(0), A.stride(1), N, 1, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8,
            GROUP_SIZE_M=8, device="b200").last_stats
        assert st["path"] == "tcgen05_f16x3"
        assert device_status() == 0
        err = float((C.double() - ref).abs().max() / ref.abs().max())
        assert err <= fp32_bound(K), (K, err)


def test_tensor_core_b_padded_rows_ragged_columns(cuda):
    """Row-major B viewed out of wider padded rows (row stride a multiple of 4 elements, 16-byte
    aligned, N = 258 not a multiple of 4): the B split loads four columns per float4 and the
    last, partial quad element by element."""
    torch = cuda
    M, N, K = 512, 258, 300
    A = torch.rand(M, K, device="cuda") * 2 - 1
    B = (torch.rand(K, 260, device="cuda") * 2 - 1)[:, :N]
    C = torch.zeros(M, N, device="cuda")
    st = Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
        A, B, C, M, N, K, A.stride(0), A.stride(1), B.stride(0), B.stride(1), C.stride(0), C.stride(1),
        BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8, device="b200").last_stats
    assert st["path"] == "tcgen05_f16x3"
    assert device_status() == 0
    ref = A.double() @ B.double()
    err = float((C.double() - ref).abs().max() / ref.abs().max())
    assert err <= fp32_bound(K), err


@pytest.mark.parametrize("K", [257, 1004])
def test_tensor_core_transposed_operands_odd_k(cuda, K):
    """A and B given as transposes (unit stride along M and along K): A goes through the
    strided (tile) split and B through the row split (B^T rows are contiguous), both
    zero-filled up to the next multiple of 8 k-values; C written through a transposed view."""
    torch = cuda
    M, N = 384, 256
    A = (torch.rand(K, M, device="cuda") * 2 - 1).t()     # stride_am = 1, stride_ak = M
    B = (torch.rand(N, K, device="cuda") * 2 - 1).t()     # stride_bk = 1, stride_bn = K
    C = torch.zeros(N, M, device="cuda").t()              # stride_cm = 1, stride_cn = M
    st = Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
        A, B, C, M, N, K, A.stride(0), A.stride(1), B.stride(0), B.stride(1), C.stride(0), C.stride(1),
        BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8, device="b200").last_stats
    assert st["path"] == "tcgen05_f16x3"
    assert device_status() == 0
    ref = A.double() @ B.double()
    err = float((C.double() - ref).abs().max() / ref.abs().max())
    assert err <= fp32_bound(K), err


def test_tensor_core_wide_dynamic_range(cuda):
    """Rows of A and columns of B spread over 2^-60 .. 2^60, far outside fp16's range: the
    per-chunk power-of-two scaling keeps every element at fp32 level relative to its own row's
    and column's magnitude (a single scale per matrix would flush the small ones to zero).
    Dividing C by the row and column powers of two (exact) gives the product of the unscaled
    U[-1, 1] operands, checked at the usual fp32-level normalised error."""
    torch = cuda
    M, N, K = 640, 768, 700
    g = torch.Generator(device="cuda").manual_seed(60)
    ra = torch.exp2(torch.randint(-60, 61, (M, 1), device="cuda", generator=g).float())
    cb = torch.exp2(torch.randint(-60, 61, (1, N), device="cuda", generator=g).float())
    A = (torch.rand(M, K, device="cuda", generator=g) * 2 - 1) * ra
    B = (torch.rand(K, N, device="cuda", generator=g) * 2 - 1) * cb
    C = torch.empty(M, N, device="cuda")
    st = Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
        A, B, C, M, N, K, K, 1, N, 1, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8,
        device="b200").last_stats
    assert st["path"] == "tcgen05_f16x3"
    assert device_status() == 0
    exact = (A / ra).double() @ (B / cb).double()
    got = C.double() / (ra.double() * cb.double())
    err = float((got - exact).abs().max() / exact.abs().max())
    assert err <= fp32_bound(K), err


def test_tensor_core_non_finite_operands(cuda):
    """inf and nan inputs keep IEEE semantics on the tensor-core path: rows of A and columns of B
    whose chunks hold one are recomputed in fp32 after the GEMM (a split product would give nan
    for inf times an exactly representable value), every other element is unaffected."""
    torch = cuda
    M, N, K = 512, 384, 1000
    g = torch.Generator(device="cuda").manual_seed(61)
    A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1
    B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
    B[5, :] = 1.0                                   # exactly representable: its low halves are zero
    A[3, 5] = float("inf")
    A[100, 999] = float("-inf")
    A[200, 7] = float("inf")
    A[200, 8] = float("-inf")                        # inf + -inf: nan
    B[300, 7] = float("nan")
    C = torch.empty(M, N, device="cuda")
    st = Launcher(matmul_kernel, (triton.cdiv(M, 8) * triton.cdiv(N, 64),))(
        A, B, C, M, N, K, K, 1, N, 1, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8,
        device="b200").last_stats
    assert st["path"] == "tcgen05_f16x3"
    assert device_status() == 0
    exact = (A.double() @ B.double()).cpu().numpy()
    got = C.double().cpu().numpy()
    np.testing.assert_array_equal(np.isnan(got), np.isnan(exact))
    np.testing.assert_array_equal(np.isposinf(got), np.isposinf(exact))
    np.testing.assert_array_equal(np.isneginf(got), np.isneginf(exact))
    fin = np.isfinite(exact)
    assert fin.sum() > 0.9 * fin.size
    err = float(np.abs(got[fin] - exact[fin]).max() / np.abs(exact[fin]).max())
    assert err <= fp32_bound(K), err
