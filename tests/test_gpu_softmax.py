"""Fused row softmax on the B200 (examples/kernels.py:60-76).

Tolerance: relative error <= 1e-5 per element against the oracle (which
reproduces the emulator bit for bit) and against float64, as the hot-path
contract states for softmax; the reference's own test uses rtol 2e-5,
atol 1e-6 against numpy (tests/test_kernels.py:16-22).  With qpu_rounding=True
the kernel runs the QPU float model and must match the emulator bit for bit.
"""

import numpy as np
import pytest

from conftest import golden_ids, goldens, sha256
from oracle import oracle as O
from piton_b200 import workloads as W
from piton_b200.kernels import softmax_kernel

pytestmark = pytest.mark.gpu
SOFTMAX = goldens("softmax_")
RTOL = 1e-5


def run(x, block, out=None, rows=None):
    m, n = x.shape
    y = np.zeros_like(x) if out is None else out
    softmax_kernel[(rows or m,)](y, x, n, n, n, BLOCK_SIZE=block, device="b200")
    return y


def rel_err(a, b):
    b = np.asarray(b, np.float64)
    return float((np.abs(a - b) / np.maximum(np.abs(b), 1e-37)).max())


@pytest.mark.parametrize("rows,cols,block", [(4, 64, 64), (3, 100, 128), (5, 16, 16)])
def test_reference_shapes(cuda, rows, cols, block):
    x = np.random.default_rng(42).standard_normal((rows, cols)).astype(np.float32)
    y = run(x, block)
    e = np.exp(x - x.max(1, keepdims=True))
    np.testing.assert_allclose(y, e / e.sum(1, keepdims=True), rtol=2e-5, atol=1e-6)


@pytest.mark.parametrize("g", SOFTMAX, ids=golden_ids(SOFTMAX))
def test_matches_emulator_golden(cuda, g):
    m = g.meta
    x = W.softmax_input(1823 if m["n"] == 781 else m["m"], m["n"], m["seed"])[:m["m"]]
    y = run(x, m["block"])
    ref = O.qpu_softmax(x, m["block"])
    assert rel_err(y, ref) <= RTOL
    assert np.all(y[np.isneginf(x)] == 0)


@pytest.mark.parametrize("g", SOFTMAX, ids=golden_ids(SOFTMAX))
def test_qpu_rounding_bit_exact_with_emulator(cuda, g):
    """qpu_rounding=True: the reference's program on the QPU float model, every output word equal
    to the emulator's (the fixture holds the SHA-256 of its output)."""
    m = g.meta
    x = W.softmax_input(1823 if m["n"] == 781 else m["m"], m["n"], m["seed"])[:m["m"]]
    y = np.zeros_like(x)
    softmax_kernel[(x.shape[0],)](y, x, x.shape[1], x.shape[1], x.shape[1], BLOCK_SIZE=m["block"],
                                  device="b200", qpu_rounding=True)
    assert sha256(y) == m["sha_out"]


@pytest.mark.parametrize("rows,cols,block", [(7, 5, 8), (9, 16, 16), (33, 100, 128), (5, 300, 128),
                                             (3, 2000, 2048)])
def test_qpu_rounding_matches_oracle(cuda, rows, cols, block):
    """Ragged rows, BLOCK below 16 and below the row, all--inf and single-finite rows, signed
    zeros and large values: bit for bit with the oracle's restatement."""
    rng = np.random.default_rng(rows * cols)
    x = (rng.standard_normal((rows, cols)) * 8).astype(np.float32)
    x[0, :] = -np.inf
    x[1, :] = -np.inf
    x[1, cols // 2] = 3.0
    x[2, ::3] = -0.0
    x[-1, 0] = 80.0
    y = np.full((rows, cols), 9.0, np.float32)
    softmax_kernel[(rows,)](y, x, cols, cols, cols, BLOCK_SIZE=block, device="b200", qpu_rounding=True)
    ref = O.qpu_softmax(x, block)
    n = min(cols, block)
    np.testing.assert_array_equal(y[:, :n].view(np.uint32), ref[:, :n].view(np.uint32))
    assert np.all(y[:, n:] == 9.0)


def test_config_1823x781_vs_float64(cuda):
    x = W.softmax_input(1823, 781, 0)
    y = run(x, 1024)
    assert rel_err(y, O.softmax_f64(x)) <= RTOL
    np.testing.assert_allclose(y.sum(1), 1.0, atol=2e-6)


@pytest.mark.parametrize("n", [256, 1024, 4096, 16384, 40000])
def test_sweep_widths(cuda, n):
    x = W.softmax_input(64, n, seed=n)
    y = run(x, 1 << (n - 1).bit_length())
    assert rel_err(y, O.softmax_f64(x)) <= RTOL


def test_block_smaller_than_row_and_strided_rows(cuda):
    torch = cuda
    x = torch.randn(8, 300, device="cuda")
    out = torch.full((8, 300), 5.0, device="cuda")
    softmax_kernel[(8,)](out, x, 300, 300, 300, BLOCK_SIZE=128, device="b200")   # only 128 columns
    ref = torch.softmax(x[:, :128].double(), 1).float()
    torch.testing.assert_close(out[:, :128], ref, rtol=RTOL, atol=1e-7)
    assert bool((out[:, 128:] == 5.0).all())
    # padded rows: stride 260 floats (16-byte aligned), 250 live columns
    buf = torch.randn(6, 260, device="cuda")
    o = torch.zeros(6, 260, device="cuda")
    softmax_kernel[(6,)](o, buf, 260, 260, 250, BLOCK_SIZE=256, device="b200")
    torch.testing.assert_close(o[:, :250], torch.softmax(buf[:, :250].double(), 1).float(), rtol=RTOL, atol=1e-7)
    assert bool((o[:, 250:] == 0).all())


def test_in_place(cuda):
    torch = cuda
    x = torch.randn(33, 1000, device="cuda")
    ref = torch.softmax(x.double(), 1).float()
    softmax_kernel[(33,)](x, x, 1000, 1000, 1000, BLOCK_SIZE=1024, device="b200")
    torch.testing.assert_close(x, ref, rtol=RTOL, atol=1e-7)
