"""Vector add and LayerNorm on the B200 through kernel[grid](..., device="b200").

Mirrors tests/test_vector_add.py of the reference (guard band after n proves
the mask) and adds: the emulator golden (bit-exact in the QPU rounding mode,
<= 1 ulp in IEEE mode), the configuration size n = 65,537 and the sweep sizes
checked against numpy's IEEE float32 add (bit-exact).
"""

import numpy as np
import pytest

import piton_b200 as triton
from conftest import golden_ids, goldens, max_ulp
from oracle import oracle as O
from piton_b200 import workloads as W
from piton_b200.kernels import add_kernel, layernorm_kernel

pytestmark = pytest.mark.gpu
ADD = goldens("add_")


@pytest.mark.parametrize("n,block", [(64, 64), (1000, 64), (4096, 256), (37, 16), (16, 16), (65537, 256)])
def test_vector_add_guard_band(cuda, n, block):
    rng = np.random.default_rng(0)
    x = rng.standard_normal(n).astype(np.float32)
    y = rng.standard_normal(n).astype(np.float32)
    out = np.full(n + 16, 7.0, dtype=np.float32)
    grid = lambda meta: (triton.cdiv(n, meta["BLOCK_SIZE"]),)
    add_kernel[grid](x, y, out, n, BLOCK_SIZE=block, device="b200")
    np.testing.assert_array_equal(out[:n], x + y)          # IEEE round-to-nearest: numpy's bits
    assert np.all(out[n:] == 7.0)


@pytest.mark.parametrize("g", ADD, ids=golden_ids(ADD))
def test_add_matches_emulator_golden(cuda, g):
    m = g.meta
    x, y = W.vector_add(m["n"], m["seed"])
    out = np.zeros(m["n"], np.float32)
    add_kernel[(triton.cdiv(m["n"], m["block"]),)](x, y, out, m["n"], BLOCK_SIZE=m["block"], device="b200",
                                                  qpu_rounding=True)
    ref = O.qpu_add(x, y)
    np.testing.assert_array_equal(out.view(np.uint32), ref.view(np.uint32))
    if "out" in g:
        np.testing.assert_array_equal(out.view(np.uint32), g["out"].view(np.uint32))
    out2 = np.zeros_like(out)
    add_kernel[(triton.cdiv(m["n"], m["block"]),)](x, y, out2, m["n"], BLOCK_SIZE=m["block"], device="b200")
    assert max_ulp(out2, ref) <= 1                          # RN vs the QPU's truncation


def test_partial_grid_writes_only_launched_programs(cuda):
    n, block = 1000, 64
    x, y = W.vector_add(n, 1)
    out = np.full(n, -3.0, np.float32)
    add_kernel[(5,)](x, y, out, n, BLOCK_SIZE=block, device="b200")
    np.testing.assert_array_equal(out[:320], x[:320] + y[:320])
    assert np.all(out[320:] == -3.0)


def test_misaligned_and_odd_views_take_the_scalar_path(cuda):
    torch = cuda
    n = 10001
    base = torch.randn(3 * n + 3, device="cuda")
    x, y, out = base[1:n + 1], base[n + 2:2 * n + 2], torch.zeros(n + 1, device="cuda")[1:]
    add_kernel[(triton.cdiv(n, 256),)](x, y, out, n, BLOCK_SIZE=256, device="b200")
    torch.testing.assert_close(out, x + y, rtol=0, atol=0)


@pytest.mark.parametrize("logn", [20, 24])
def test_sweep_sizes_bit_exact_vs_numpy(cuda, logn):
    n = 1 << logn
    x, y = W.vector_add(n, logn)
    out = np.empty(n, np.float32)
    add_kernel[(triton.cdiv(n, 1024),)](x, y, out, n, BLOCK_SIZE=1024, device="b200")
    np.testing.assert_array_equal(out, x + y)


def test_qpu_rounding_special_values(cuda):
    f = np.float32
    x = np.array([np.inf, -np.inf, np.nan, 1e-40, 3e38, 1.0, 1.0, 0.0], f)
    y = np.array([-np.inf, np.inf, 1.0, 0.0, 3e38, 2.0 ** -24, -(2.0 ** -25), -0.0], f)
    out = np.zeros_like(x)
    add_kernel[(1,)](x, y, out, x.size, BLOCK_SIZE=16, device="b200", qpu_rounding=True)
    np.testing.assert_array_equal(out.view(np.uint32), O.qpu_add(x, y).view(np.uint32))


def test_bad_buffer_size_is_rejected_before_launch(cuda):
    x = np.zeros(100, np.float32)
    with pytest.raises(ValueError):
        add_kernel[(1,)](x, x, np.zeros(50, np.float32), 100, BLOCK_SIZE=128, device="b200")


@pytest.mark.parametrize("block,n", [(256, 256), (256, 200), (128, 100), (128, 127), (2048, 1500)])
def test_layernorm(cuda, block, n):
    rng = np.random.default_rng(7)
    rows = 3
    x = (rng.standard_normal((rows, block)) * 2 + 1).astype(np.float32)
    out = np.full(rows * block, np.nan, np.float32)
    layernorm_kernel[(rows,)](x.ravel(), out, n, 1e-5, BLOCK=block, device="b200")
    xs = x[:, :n].astype(np.float64)
    d = xs - xs.mean(axis=1, keepdims=True)
    ref = d / np.sqrt((d * d).mean(axis=1, keepdims=True) + 1e-5)
    out = out.reshape(rows, block)
    np.testing.assert_allclose(out[:, :n], ref, rtol=1e-4, atol=1e-4)     # tests/test_reroll_reduce.py:227
    assert np.isnan(out[:, n:]).all()
