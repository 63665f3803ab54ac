"""The reference's benchmark suite cases (perf/suite.py:150-350, run by perf/test_perf_suite.py)
through kernel[grid](..., device="b200"), at the suite's Raspberry Pi sizes (vectors of
262144 elements, 256 x 256 matrices, 1800 images), with its inputs and tolerances.

Inputs come from the 32-bit linear congruential generator the suite uses (multiplier
1664525, increment 1013904223, the Numerical Recipes constants): floats are the top 24 bits
of each output scaled to [-1, 1), then to the case's range; every case draws its buffers
from seeds 2 x 1000003, 3 x 1000003, ... in argument order.  The Mandelbrot and compute-peak
cases measure the Pi's ALU and are not operators of this backend."""

import numpy as np
import pytest

from piton_b200 import kernels as K

gpu = pytest.mark.gpu

VEC, MAT, DENSE_M = 262144, 256, 1800
LCG_MUL, LCG_INC, MASK = 1664525, 1013904223, 0xFFFFFFFF


def lcg_u32(n, seed):
    """The first n states after `seed` of s <- (1664525 s + 1013904223) mod 2^32: a scalar
    loop for 1024 states, then jumps of 1024 steps applied to whole blocks."""
    blk = 1024
    s = seed & MASK
    head = np.empty(min(n, blk), np.uint64)
    for i in range(len(head)):
        s = (LCG_MUL * s + LCG_INC) & MASK
        head[i] = s
    jump_a, jump_c = 1, 0                      # s -> jump_a s + jump_c advances 1024 steps
    for _ in range(blk):
        jump_a, jump_c = (LCG_MUL * jump_a) & MASK, (LCG_MUL * jump_c + LCG_INC) & MASK
    parts, cur, have = [head], head, len(head)
    while have < n:
        cur = (np.uint64(jump_a) * cur + np.uint64(jump_c)) & np.uint64(MASK)
        parts.append(cur)
        have += len(cur)
    return np.concatenate(parts)[:n].astype(np.uint32)


class Draws:
    """Buffers of one case, seeds 2 x 1000003, 3 x 1000003, ... in the order they are drawn."""

    def __init__(self):
        self.k = 1

    def seed(self):
        self.k += 1
        return 1000003 * self.k

    def floats(self, n, lo=-1.0, hi=1.0):
        u = lcg_u32(n, self.seed())
        x = (u >> np.uint32(8)).astype(np.float32) * np.float32(2.0 ** -23) - np.float32(1.0)
        return x * np.float32((hi - lo) / 2) + np.float32((hi + lo) / 2)

    def ints(self, n, shift=0, or_mask=0):
        return (lcg_u32(n, self.seed()).view(np.int32) >> shift) | np.int32(or_mask)


def check(out, ref, rtol, atol):
    np.testing.assert_allclose(out.astype(np.float64), ref, rtol=rtol, atol=atol)


ELEMENTWISE = [
    # name, kernel, inputs, scalar, constants, op, lo, hi, rtol, atol
    ("copy", K.copy_kernel, 1, None, {"BLOCK": 256}, lambda x: x, -1, 1, 1e-6, 1e-6),
    ("add", K.add_kernel, 2, None, {"BLOCK_SIZE": 256}, lambda x, y: x + y, -1, 1, 1e-6, 1e-6),
    ("mul", K.mul_kernel, 2, None, {"BLOCK": 256}, lambda x, y: x * y, -1, 1, 1e-6, 1e-6),
    ("fma", K.fma_kernel, 2, 1.5, {"BLOCK": 256}, lambda x, y: x * 1.5 + y, -1, 1, 1e-6, 1e-6),
    ("scaled_relu", K.scaled_relu_kernel, 1, 0.5, {"BLOCK": 256}, lambda x: np.where(x > 0, x * 0.5, 0.0), -1, 1,
     1e-6, 1e-6),
    ("exp", K.sfu_kernel, 1, None, {"OP": 4, "BLOCK": 256}, np.exp, -8, 8, 4e-6, 1e-30),
    ("exp2", K.sfu_kernel, 1, None, {"OP": 0, "BLOCK": 256}, np.exp2, -8, 8, 4e-6, 1e-30),
    ("log", K.log_kernel, 1, None, {"BLOCK": 256}, np.log, 0.01, 100, 4e-6, 4e-7),
    ("log2", K.sfu_kernel, 1, None, {"OP": 1, "BLOCK": 256}, np.log2, 0.01, 100, 4e-6, 4e-7),
    ("recip", K.sfu_kernel, 1, None, {"OP": 2, "BLOCK": 256}, lambda x: 1.0 / x, 0.01, 100, 4e-6, 1e-30),
    ("rsqrt", K.sfu_kernel, 1, None, {"OP": 3, "BLOCK": 256}, lambda x: 1.0 / np.sqrt(x), 0.01, 100, 4e-6, 1e-30),
    ("sqrt", K.sfu_kernel, 1, None, {"OP": 5, "BLOCK": 256}, np.sqrt, 0.01, 100, 4e-6, 1e-30),
]


@gpu
@pytest.mark.parametrize("case", ELEMENTWISE, ids=[c[0] for c in ELEMENTWISE])
def test_elementwise_and_sfu_cases(cuda, case):
    name, kern, inputs, scalar, cons, op, lo, hi, rtol, atol = case
    d = Draws()
    xs = [d.floats(VEC, lo, hi) for _ in range(inputs)]
    out = np.zeros(VEC, np.float32)
    args = xs + [out, VEC] + ([float(scalar)] if scalar is not None else [])
    kern[(VEC // 256,)](*args, **cons, device="b200")
    check(out, op(*[x.astype(np.float64) for x in xs]), rtol, atol)


@gpu
def test_idiv_case(cuda):
    d = Draws()
    x = d.ints(VEC)
    y = d.ints(VEC, shift=8, or_mask=1)                 # nonzero divisors of varied size
    q = np.zeros(VEC, np.int32)
    r = np.zeros(VEC, np.int32)
    K.idiv_kernel[(VEC // 256,)](x, y, q, r, VEC, BLOCK=256, device="b200")
    x64, y64 = x.astype(np.int64), y.astype(np.int64)
    want_q = np.sign(x64) * np.sign(y64) * (np.abs(x64) // np.abs(y64))   # C division: toward zero
    np.testing.assert_array_equal(q, want_q.astype(np.int32))
    np.testing.assert_array_equal(r, (x64 - want_q * y64).astype(np.int32))


@gpu
@pytest.mark.parametrize("name,kern,op,rtol", [("row_sum", K.row_sum_kernel, np.sum, 1e-5),
                                               ("row_max", K.row_max_kernel, np.max, 0.0)])
def test_row_reduce_cases(cuda, name, kern, op, rtol):
    x = Draws().floats(MAT * MAT).reshape(MAT, MAT)
    out = np.zeros(MAT, np.float32)
    kern[(MAT // 4,)](x, out, MAT, MAT, BLOCK_M=4, BLOCK_N=64, device="b200")
    check(out, op(x.astype(np.float64), axis=1), rtol, 1e-5)


@gpu
def test_transpose_case(cuda):
    x = Draws().floats(MAT * MAT).reshape(MAT, MAT)
    out = np.zeros(MAT * MAT, np.float32)
    K.transpose_kernel[((MAT // 16) ** 2,)](x, out, MAT, MAT, MAT, MAT, BLOCK_M=16, BLOCK_N=16, device="b200")
    np.testing.assert_array_equal(out, x.T.ravel())


@gpu
def test_softmax_case(cuda):
    x = Draws().floats(MAT * MAT, -4.0, 4.0).reshape(MAT, MAT)
    out = np.zeros((MAT, MAT), np.float32)
    K.softmax_kernel[(MAT,)](out, x, MAT, MAT, MAT, BLOCK_SIZE=MAT, device="b200")
    xd = x.astype(np.float64)
    e = np.exp(xd - xd.max(axis=1, keepdims=True))
    check(out, e / e.sum(axis=1, keepdims=True), 2e-5, 1e-8)


@gpu
@pytest.mark.parametrize("bk", [4, 8])
def test_matmul_cases(cuda, bk):
    """matmul_8x64x4 and matmul_8x64x8: [256, 256] @ [256, 256] with K a launch constant."""
    n = kk = MAT
    d = Draws()
    a = d.floats(n * kk).reshape(n, kk)
    b = d.floats(kk * n).reshape(kk, n)
    c = np.zeros((n, n), np.float32)
    grid = (((n + 7) // 8) * ((n + 63) // 64),)
    K.matmul_kernel[grid](a, b, c, n, n, kk, kk, 1, n, 1, n, 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64,
                          BLOCK_SIZE_K=bk, GROUP_SIZE_M=4, device="b200")
    check(c, a.astype(np.float64) @ b.astype(np.float64), 1e-3, 2e-4 * kk)


@gpu
def test_dense_relu_case(cuda):
    """The digits network's first layer over 1800 rows: ReLU(x W + b), 64 -> 128."""
    m, n_in, n_out = DENSE_M, 64, 128
    d = Draws()
    x = d.floats(m * n_in, 0.0, 1.0).reshape(m, n_in)
    w = d.floats(n_in * n_out, -0.3, 0.3).reshape(n_in, n_out)
    bias = d.floats(n_out, -0.1, 0.1)
    y = np.zeros((m, n_out), np.float32)
    K.dense_layer_kernel[((m // 4) * (n_out // 64),)](x, w, bias, y, m, N=n_out, K=n_in, BLOCK_SIZE_M=4,
                                                      BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=1,
                                                      ADD_BIAS=True, RELU=True, device="b200")
    want = np.maximum(x.astype(np.float64) @ w.astype(np.float64) + bias, 0)
    check(y, want, 1e-4, 1e-4)


def test_lcg_matches_the_recurrence():
    """No GPU needed: the block jump-ahead equals the plain recurrence."""
    s, want = 12345, []
    for _ in range(3000):
        s = (LCG_MUL * s + LCG_INC) & MASK
        want.append(s)
    np.testing.assert_array_equal(lcg_u32(3000, 12345), np.array(want, np.uint32))
