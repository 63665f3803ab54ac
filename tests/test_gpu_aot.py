"""AOT launchers (piton_b200.tools.compile) on the B200: the emitted C, built
into a shared object here and called through ctypes with device pointers,
gives the same bits as the ``kernel[grid](..., device="b200")`` launch of the
same operator (both reach the same entry point), and the same answers as the
oracle where the operator is exact."""

import ctypes as C
import os
import shutil
import subprocess

import numpy as np
import pytest

import piton_b200 as triton
from aot_cases import CASES
from oracle import oracle as O
from piton_b200 import kernels as K
from piton_b200 import workloads as W
from piton_b200.runtime.launcher import offset_ptr
from piton_b200.tools import compile as aot

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KERNELS = os.path.join(ROOT, "piton_b200", "kernels.py")
LIBDIR = os.path.join(ROOT, "piton_b200")
UINT32_MAX = 0xFFFFFFFF


@pytest.fixture(scope="module")
def launchers(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    out = tmp_path_factory.mktemp("aot_gpu")
    srcs, types = [], {}
    for name, kern, sig, cons, opts in CASES:
        aot.compile_kernel(KERNELS, kern, sig, cons, name, str(out), **opts)
        srcs.append(str(out / f"{name}.c"))
        types[name] = aot.ctypes_args(aot.kernel_params(getattr(K, kern)), sig)
    so = out / "libaot.so"
    r = subprocess.run([cc, "-std=c99", "-O2", "-shared", "-fPIC", "-I", os.path.join(ROOT, "include"), "-I",
                        str(out), *srcs, "-o", str(so), "-L", LIBDIR, "-lpiton_b200", f"-Wl,-rpath,{LIBDIR}"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    lib = C.CDLL(str(so))

    def launch(name, grid, **fields):
        T = types[name]
        args = T(**fields)
        f = getattr(lib, f"{name}_launch")
        f.restype = C.c_uint32
        f.argtypes = [C.POINTER(T), C.c_uint, C.c_uint, C.c_uint]
        g = tuple(grid) + (1,) * (3 - len(grid))
        return f(C.byref(args), *g)
    return launch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_add_and_elapsed_time(cuda, launchers):
    torch = cuda
    n = 65537
    x, y = W.vector_add(n, 0)
    tx, ty, to = dev(torch, x), dev(torch, y), torch.zeros(n, device="cuda")
    us = launchers("aot_add", (triton.cdiv(n, 256),), x_ptr=tx.data_ptr(), y_ptr=ty.data_ptr(),
                   output_ptr=to.data_ptr(), n_elements=n)
    assert 0 <= us < UINT32_MAX
    np.testing.assert_array_equal(to.cpu().numpy(), x + y)
    # QPU rounding: the emulator's bits
    m = 1000
    to2 = torch.zeros(m, device="cuda")
    launchers("aot_add_qpu", (triton.cdiv(m, 64),), x_ptr=tx.data_ptr(), y_ptr=ty.data_ptr(),
              output_ptr=to2.data_ptr(), n_elements=m)
    np.testing.assert_array_equal(bits(to2.cpu().numpy()), bits(O.qpu_add(x[:m], y[:m])))


def test_softmax_same_bits_as_the_launch(cuda, launchers):
    torch = cuda
    x = W.softmax_input(1823, 781, 0)
    want = np.zeros_like(x)
    K.softmax_kernel[(1823,)](want, x, 781, 781, 781, BLOCK_SIZE=1024, device="b200")
    tx, to = dev(torch, x), torch.zeros(1823, 781, device="cuda")
    assert launchers("aot_softmax", (1823,), output_ptr=to.data_ptr(), input_ptr=tx.data_ptr(),
                     input_row_stride=781, output_row_stride=781, n_cols=781) < UINT32_MAX
    np.testing.assert_array_equal(bits(to.cpu().numpy()), bits(want))


def test_matmul_constant_k_same_bits_as_the_launch(cuda, launchers):
    torch = cuda
    M = N = Kd = 512
    a, b = W.matmul_inputs(M, N, Kd, 1)
    want = np.zeros((M, N), np.float32)
    grid = (triton.cdiv(M, 8) * triton.cdiv(N, 64),)
    K.matmul_kernel[grid](a, b, want, M, N, Kd, Kd, 1, N, 1, N, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64,
                          BLOCK_SIZE_K=4, GROUP_SIZE_M=4, device="b200")
    ta, tb, tc = dev(torch, a), dev(torch, b), torch.zeros(M, N, device="cuda")
    assert launchers("aot_matmul", grid, a_ptr=ta.data_ptr(), b_ptr=tb.data_ptr(), c_ptr=tc.data_ptr(), M=M, N=N,
                     stride_am=Kd, stride_bk=N, stride_cm=N) < UINT32_MAX
    np.testing.assert_array_equal(bits(tc.cpu().numpy()), bits(want))
    # QPU rounding, K = 64: the oracle's bits
    a2, b2 = W.matmul_inputs(72, 100, 64, 2)
    ta2, tb2, tc2 = dev(torch, a2), dev(torch, b2), torch.zeros(72, 100, device="cuda")
    launchers("aot_matmul_qpu", (triton.cdiv(72, 8) * triton.cdiv(100, 64),), a_ptr=ta2.data_ptr(),
              b_ptr=tb2.data_ptr(), c_ptr=tc2.data_ptr(), M=72, N=100, stride_am=64, stride_bk=100, stride_cm=100)
    np.testing.assert_array_equal(bits(tc2.cpu().numpy()), bits(O.qpu_matmul(a2, b2)))


def test_matmul_runtime_strides_negative_c(cuda, launchers):
    torch = cuda
    M, N, Kd = 1000, 777, 513
    a, b = W.matmul_inputs(M, N, Kd, 3)
    grid = (triton.cdiv(M, 8) * triton.cdiv(N, 64),)
    want = np.zeros((M, N), np.float32)
    K.matmul_kernel[grid](a, b, offset_ptr(want, (M - 1) * N), M, N, Kd, Kd, 1, N, 1, -N, 1, BLOCK_SIZE_M=8,
                          BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8, device="b200")
    ta, tb, tc = dev(torch, a), dev(torch, b), torch.zeros(M, N, device="cuda")
    launchers("aot_matmul_rt", grid, a_ptr=ta.data_ptr(), b_ptr=tb.data_ptr(),
              c_ptr=tc.data_ptr() + 4 * (M - 1) * N, M=M, N=N, K=Kd, stride_am=Kd, stride_ak=1, stride_bk=N,
              stride_bn=1, stride_cm=-N, stride_cn=1)
    got = tc.cpu().numpy()
    np.testing.assert_array_equal(bits(got), bits(want))
    ref = (a.astype(np.float64) @ b.astype(np.float64))[::-1]
    assert np.abs(got - ref).max() / np.abs(ref).max() <= 1e-7 * np.sqrt(Kd) + 4e-6


def test_attention_same_bits_as_the_launch(cuda, launchers):
    torch = cuda
    heads, S, D = 16, 256, 64
    q, k, v = W.attention_inputs(heads, S, D, 0)
    want = np.zeros_like(q)
    grid = (triton.cdiv(S, 2), heads)
    K.attn_fwd_kernel[grid](q, k, v, want, 0.125, S * D, D, S * D, D, 1, S * D, D, S * D, D, S, HEAD_DIM=D,
                            BLOCK_M=2, BLOCK_N=16, CAUSAL=True, EVEN_N=True, device="b200")
    tq, tk, tv, to = dev(torch, q), dev(torch, k), dev(torch, v), torch.zeros(heads, S, D, device="cuda")
    assert launchers("aot_attn", grid, Q=tq.data_ptr(), K=tk.data_ptr(), V=tv.data_ptr(), Out=to.data_ptr(),
                     sm_scale=0.125, stride_qh=S * D, stride_kh=S * D, stride_vh=S * D, stride_oh=S * D) < UINT32_MAX
    np.testing.assert_array_equal(bits(to.cpu().numpy()), bits(want))


def test_qpu_softmax_attention_and_sigmoid_launchers(cuda, launchers):
    """The QPU-rounding softmax and attention launchers give the oracle's (the emulator's) bits;
    the sigmoid launcher the kernel[grid] launch's."""
    torch = cuda
    x = W.softmax_input(64, 781, 1)
    tx, to = dev(torch, x), torch.zeros(64, 781, device="cuda")
    assert launchers("aot_softmax_qpu", (64,), output_ptr=to.data_ptr(), input_ptr=tx.data_ptr(),
                     input_row_stride=781, output_row_stride=781, n_cols=781) < UINT32_MAX
    np.testing.assert_array_equal(bits(to.cpu().numpy()), bits(O.qpu_softmax(x, 1024)))
    heads, S, D = 2, 256, 64
    q, k, v = W.attention_inputs(heads, S, D, 3)
    tq, tk, tv, ta = dev(torch, q), dev(torch, k), dev(torch, v), torch.zeros(heads, S, D, device="cuda")
    assert launchers("aot_attn_qpu", (triton.cdiv(S, 2), heads), Q=tq.data_ptr(), K=tk.data_ptr(),
                     V=tv.data_ptr(), Out=ta.data_ptr(), sm_scale=0.125, stride_qh=S * D, stride_kh=S * D,
                     stride_vh=S * D, stride_oh=S * D) < UINT32_MAX
    np.testing.assert_array_equal(bits(ta.cpu().numpy()), bits(O.qpu_attention(q, k, v, True, sm_scale=0.125)))
    n = 1000
    xs = np.linspace(-12, 12, n, dtype=np.float32)
    want = np.zeros(n, np.float32)
    K.sigmoid_kernel[(triton.cdiv(n, 256),)](xs, want, n, BLOCK=256, device="b200")
    ts, tso = dev(torch, xs), torch.zeros(n, device="cuda")
    assert launchers("aot_sigmoid", (triton.cdiv(n, 256),), x_ptr=ts.data_ptr(), out_ptr=tso.data_ptr(),
                     n=n) < UINT32_MAX
    np.testing.assert_array_equal(bits(tso.cpu().numpy()), bits(want))


def test_integer_and_life_launchers_are_exact(cuda, launchers):
    torch = cuda
    rng = np.random.default_rng(9)
    n = 50000
    x = rng.integers(-2**31, 2**31, n, dtype=np.int64).astype(np.int32)
    y = rng.integers(-2**31, 2**31, n, dtype=np.int64).astype(np.int32)
    y[y == 0] = 7
    tx, ty = dev(torch, x), dev(torch, y)
    tq, tr = torch.zeros(n, dtype=torch.int32, device="cuda"), torch.zeros(n, dtype=torch.int32, device="cuda")
    launchers("aot_idiv", (triton.cdiv(n, 256),), x_ptr=tx.data_ptr(), y_ptr=ty.data_ptr(), q_ptr=tq.data_ptr(),
              r_ptr=tr.data_ptr(), n=n)
    wq, wr = O.idiv_c(x, y, True)
    np.testing.assert_array_equal(bits(tq.cpu().numpy()), wq)
    np.testing.assert_array_equal(bits(tr.cpu().numpy()), wr)
    cells = (rng.random((40, 128)) < 0.35).astype(np.int32)
    w = O.pack_bits(cells)
    src, dst = dev(torch, w.view(np.int32)), torch.zeros(w.shape, dtype=torch.int32, device="cuda")
    launchers("aot_life_bits", (triton.cdiv(w.shape[1], 16), triton.cdiv(40, 16)), src_ptr=src.data_ptr(),
              dst_ptr=dst.data_ptr(), n_rows=40, n_words=w.shape[1], stride=w.shape[1])
    got = O.unpack_bits(dst.cpu().numpy().view(np.uint32), 128)
    np.testing.assert_array_equal(got, O.life_step(cells))


def test_failed_launch_returns_uint32_max(cuda, launchers):
    torch = cuda
    t = torch.zeros(16, device="cuda")
    us = launchers("aot_matmul", (1,), a_ptr=t.data_ptr(), b_ptr=t.data_ptr(), c_ptr=t.data_ptr(), M=-1, N=4,
                   stride_am=1, stride_bk=1, stride_cm=1)
    assert us == UINT32_MAX
    from piton_b200.runtime.cuda import lib
    assert b"negative shape" in lib().piton_b200_last_error()
