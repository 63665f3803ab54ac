"""The remaining example operators on the B200: element-wise ops, exact integer
division, row reductions, transpose and the three Game of Life kernels.

Bit-exact where the operator is exact (idiv, Life, copy, transpose, row max,
mul / fma / scaled ReLU against numpy in IEEE mode and against the emulator in
QPU rounding mode); the math functions are checked against float64 within the
accuracy the reference's ALU sequences have (tests/test_tiles.py).
"""

import numpy as np
import pytest

import piton_b200 as triton
from conftest import golden_ids, goldens
from oracle import oracle as O
from piton_b200 import kernels as K

pytestmark = pytest.mark.gpu
IDIV = goldens("idiv_")
LIFE = goldens("life_")
ELEM = goldens("elem_")


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.mark.parametrize("g", IDIV, ids=golden_ids(IDIV))
def test_idiv_matches_emulator(cuda, g):
    x, y = g["x"], g["y"]
    q, r = np.zeros_like(x), np.zeros_like(x)
    n = x.size
    K.idiv_kernel[(triton.cdiv(n, 64),)](x, y, q, r, n, BLOCK=64, device="b200")
    np.testing.assert_array_equal(bits(q), bits(g["q"]))
    np.testing.assert_array_equal(bits(r), bits(g["r"]))


@pytest.mark.parametrize("signed", [True, False])
def test_idiv_edges_and_random(cuda, signed):
    rng = np.random.default_rng(3)
    M32 = 0xFFFFFFFF
    e = np.array(sorted({((1 << k) + d) & M32 for k in range(33) for d in (-3, -2, -1, 0, 1, 2, 3)}), np.uint64)
    x = np.concatenate([np.repeat(e, e.size), rng.integers(0, 1 << 32, 100000, dtype=np.uint64)]).astype(np.uint32)
    y = np.concatenate([np.tile(e, e.size), rng.integers(1, 1 << 32, 100000, dtype=np.uint64)
                        >> rng.integers(0, 32, 100000).astype(np.uint64)]).astype(np.uint32)
    y[y == 0] = 1
    if signed:
        x, y = x.view(np.int32), y.view(np.int32)
    q, r = np.zeros_like(x), np.zeros_like(x)
    K.idiv_kernel[(triton.cdiv(x.size, 256),)](x, y, q, r, x.size, BLOCK=256, device="b200")
    wq, wr = O.idiv_c(x, y, signed)
    np.testing.assert_array_equal(bits(q), wq)
    np.testing.assert_array_equal(bits(r), wr)


@pytest.mark.parametrize("g", LIFE, ids=golden_ids(LIFE))
def test_life_matches_emulator(cuda, g):
    m = g.meta
    src = g["src"]
    dst = np.zeros_like(src)
    kern = {"tile": K.life_kernel, "rows": K.life_rows_kernel, "bits": K.life_bits_kernel}[m["kernel"]]
    kern[tuple(m["grid"])](src, dst, m["shape"][0], src.shape[1], src.shape[1], device="b200", **m["constants"])
    np.testing.assert_array_equal(dst, g["dst"])


@pytest.mark.parametrize("shape", [(8, 16), (13, 37), (1, 20), (5, 3), (2, 2), (40, 70), (512, 512)])
def test_life_many_generations_all_kernels(cuda, shape):
    rng = np.random.default_rng(shape[0] * 100 + shape[1])
    cells = (rng.random(shape) < 0.3).astype(np.int32)
    want = cells
    for _ in range(6):
        want = O.life_step(want)
    a, b = cells.copy(), np.zeros_like(cells)
    for _ in range(6):                                        # tiles, ping-pong buffers
        K.life_kernel[(triton.cdiv(shape[0], 4) * triton.cdiv(shape[1], 16),)](a, b, shape[0], shape[1], shape[1],
                                                                               BLOCK_R=4, BLOCK_C=16, device="b200")
        a, b = b, a
    np.testing.assert_array_equal(a, want)
    a, b = cells.copy(), np.zeros_like(cells)
    for _ in range(6):                                        # row strips
        K.life_rows_kernel[(triton.cdiv(shape[1], 64), triton.cdiv(shape[0], 32))](
            a, b, shape[0], shape[1], shape[1], ROWS=32, BLOCK=64, device="b200")
        a, b = b, a
    np.testing.assert_array_equal(a, want)
    if shape[1] % 32 == 0:
        w = O.pack_bits(cells)
        a, b = w.copy(), np.zeros_like(w)
        for _ in range(6):
            K.life_bits_kernel[(triton.cdiv(w.shape[1], 16), triton.cdiv(shape[0], 16))](
                a, b, shape[0], w.shape[1], w.shape[1], ROWS=16, BLOCK=16, device="b200")
            a, b = b, a
        np.testing.assert_array_equal(O.unpack_bits(a, shape[1]), want)


def test_life_row_stride_leaves_padding_alone(cuda):
    rng = np.random.default_rng(11)
    cells = (rng.random((10, 29)) < 0.4).astype(np.int32)
    src = np.full((10, 40), 7, np.int32)
    src[:, :29] = cells
    dst = np.full((10, 40), -5, np.int32)
    K.life_kernel[(triton.cdiv(10, 4) * triton.cdiv(29, 16),)](src, dst, 10, 29, 40, BLOCK_R=4, BLOCK_C=16,
                                                               device="b200")
    np.testing.assert_array_equal(dst[:, :29], O.life_step(cells))
    assert np.all(dst[:, 29:] == -5)


@pytest.mark.parametrize("g", ELEM, ids=golden_ids(ELEM))
def test_elementwise_qpu_mode_matches_emulator(cuda, g):
    x, y, n = g["x"], g["y"], g.meta["n"]
    out = np.zeros(n, np.float32)
    if g.meta["op"] == "elem_mul":
        K.mul_kernel[(triton.cdiv(n, 64),)](x, y, out, n, BLOCK=64, device="b200", qpu_rounding=True)
    elif g.meta["op"] == "elem_fma":
        K.fma_kernel[(triton.cdiv(n, 64),)](x, y, out, n, 0.3, BLOCK=64, device="b200", qpu_rounding=True)
    else:
        K.scaled_relu_kernel[(triton.cdiv(n, 128),)](x, out, n, 0.5, BLOCK=128, device="b200", qpu_rounding=True)
    np.testing.assert_array_equal(bits(out), bits(g["out"]))


def test_elementwise_ieee_bit_exact_vs_numpy(cuda):
    n = 300001
    rng = np.random.default_rng(5)
    x, y = rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32)
    g = (triton.cdiv(n, 256),)
    out = np.full(n + 8, 9.0, np.float32)
    K.copy_kernel[g](x, out, n, BLOCK=256, device="b200")
    np.testing.assert_array_equal(out[:n], x)
    assert np.all(out[n:] == 9.0)
    K.mul_kernel[g](x, y, out, n, BLOCK=256, device="b200")
    np.testing.assert_array_equal(out[:n], x * y)
    K.fma_kernel[g](x, y, out, n, 0.75, BLOCK=256, device="b200")
    np.testing.assert_array_equal(out[:n], x * np.float32(0.75) + y)
    K.scaled_relu_kernel[g](x, out, n, 0.5, BLOCK=256, device="b200")
    np.testing.assert_array_equal(out[:n], np.where(x > 0, x * np.float32(0.5), np.float32(0)))


@pytest.mark.parametrize("op,fn,lo,hi,ulps", [
    (0, np.exp2, -20, 20, 2), (1, np.log2, 1e-3, 1e3, 2), (2, lambda v: 1.0 / v, 0.01, 100, 1),
    (3, lambda v: 1.0 / np.sqrt(v), 1e-3, 1e3, 2), (4, np.exp, -20, 20, 2), (5, np.sqrt, 0, 1e4, 1)])
def test_sfu_ops_accuracy(cuda, op, fn, lo, hi, ulps):
    rng = np.random.default_rng(op)
    n = 100000
    x = rng.uniform(lo, hi, n).astype(np.float32)
    out = np.zeros(n, np.float32)
    K.sfu_kernel[(triton.cdiv(n, 512),)](x, out, n, OP=op, BLOCK=512, device="b200")
    exact = fn(x.astype(np.float64))
    ulp = np.spacing(np.abs(exact).astype(np.float32)).astype(np.float64)
    assert (np.abs(out - exact) / ulp).max() <= ulps + 0.5
    lg = np.zeros(n, np.float32)
    xp = rng.uniform(1e-3, 1e3, n).astype(np.float32)
    K.log_kernel[(triton.cdiv(n, 512),)](xp, lg, n, BLOCK=512, device="b200")
    np.testing.assert_allclose(lg, np.log(xp.astype(np.float64)), rtol=0, atol=4e-7 * np.log(1e3) + 1e-7)


def test_sigmoid(cuda):
    """tl.sigmoid (piton/language/core.py:787-790) element-wise: within the elementwise rel 1e-5 of
    float64 over [-30, 30] with a ragged tail, the limits at +-inf, and nan through."""
    rng = np.random.default_rng(11)
    n = 100003
    x = rng.uniform(-30, 30, n).astype(np.float32)
    x[:6] = [np.inf, -np.inf, 0.0, -0.0, np.nan, 88.0]
    out = np.full(n + 5, 7.0, np.float32)
    K.sigmoid_kernel[(triton.cdiv(n, 256),)](x, out, n, BLOCK=256, device="b200")
    exact = 1.0 / (1.0 + np.exp(-x.astype(np.float64)))
    fin = np.isfinite(x)
    np.testing.assert_allclose(out[:n][fin], exact[fin], rtol=1e-5, atol=0)
    assert out[0] == 1.0 and out[1] == 0.0 and np.isnan(out[4])
    assert np.all(out[n:] == 7.0)   # nothing past n is written


def test_row_sum_and_row_max(cuda):
    rng = np.random.default_rng(42)
    m, n = 64, 96
    x = rng.standard_normal((m, n)).astype(np.float32)
    out = np.zeros(m, np.float32)
    K.row_sum_kernel[(m // 8,)](x, out, n, n, BLOCK_M=8, BLOCK_N=32, device="b200")
    np.testing.assert_allclose(out, x.sum(1), rtol=1e-5, atol=1e-5)       # tests/test_kernels.py:42
    K.row_max_kernel[(m // 8,)](x, out, n, n, BLOCK_M=8, BLOCK_N=32, device="b200")
    np.testing.assert_array_equal(out, x.max(1))
    # the reference loads ceil(n_cols / BLOCK_N) * BLOCK_N columns, unmasked: 40 -> 64
    xs = rng.standard_normal((16, 64)).astype(np.float32)
    out2 = np.zeros(16, np.float32)
    K.row_sum_kernel[(2,)](xs, out2, 40, 64, BLOCK_M=8, BLOCK_N=32, device="b200")
    np.testing.assert_allclose(out2, xs.sum(1), rtol=1e-5, atol=1e-5)


def test_transpose(cuda):
    rng = np.random.default_rng(1)
    for nr, nc in ((64, 48), (37, 29), (1, 100)):
        x = rng.standard_normal((nr, nc)).astype(np.float32)
        out = np.full((nc, nr), 3.0, np.float32)
        tiles = triton.cdiv(nr, 16) * triton.cdiv(nc, 16)
        K.transpose_kernel[(tiles,)](x, out, nr, nc, nc, nr, BLOCK_M=16, BLOCK_N=16, device="b200")
        np.testing.assert_array_equal(out, x.T)
