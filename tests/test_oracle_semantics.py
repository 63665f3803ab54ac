"""Known-answer checks of the oracle's QPU float model (CPU only).

The values follow the rules the reference emulator documents for the VideoCore
IV ALUs (piton/qpu/emulator.py:137-150): truncation toward zero, denormals
read and written as +0, NaN read as an infinity, 0 * inf = +0, inf + -inf =
the second operand; and the ALU-only exp / reciprocal sequences
(piton/backend/lower.py:633-667, 2716-2797) against float64.
"""

import numpy as np

from oracle import oracle as O

f = np.float32


def one(op, a, b):
    return O.qpu_binary(op, np.array([a], f), np.array([b], f))[0]


def test_add_truncates_toward_zero():
    # 1 + 2^-24 is exactly halfway; truncation keeps 1, and 1 - 2^-25 truncates below 1
    assert one("fadd", 1.0, 2.0 ** -24) == f(1.0)
    assert one("fadd", 1.0, -(2.0 ** -25)) == np.nextafter(f(1.0), f(0))
    assert one("fadd", -1.0, 2.0 ** -25) == -np.nextafter(f(1.0), f(0))


def test_special_values():
    inf = np.inf
    assert one("fmul", 0.0, inf) == 0.0 and not np.signbit(one("fmul", 0.0, inf))
    assert one("fadd", inf, -inf) == -inf                       # the second operand
    assert one("fadd", -inf, inf) == inf
    assert one("fadd", np.nan, 1.0) == inf                      # NaN reads as +inf
    den = np.float32(1e-40)                                     # a denormal reads as +0
    assert one("fadd", den, 0.0) == 0.0
    assert one("fmul", 1e-30, 1e-30) == 0.0                     # underflow flushes to +0
    assert not np.signbit(one("fadd", 1.0, -1.0))               # zero results are +0
    assert one("fmul", 3e38, 10.0) == inf                       # overflow gives inf, not FLT_MAX


def test_exp_accuracy_and_limits():
    x = np.linspace(-80, 80, 20001).astype(f)
    e = O.qpu_exp(x)
    rel = np.abs(e.astype(np.float64) / np.exp(x.astype(np.float64)) - 1)
    assert rel.max() < 4e-7                                      # ~2-3 ulp, as the lowering promises
    x2 = np.linspace(-120, 120, 20001).astype(f)
    e2 = O.qpu_exp(x2, base2=True)
    rel2 = np.abs(e2.astype(np.float64) / np.exp2(x2.astype(np.float64)) - 1)
    assert rel2.max() < 4e-7
    assert O.qpu_exp(np.array([-np.inf, 200.0, -200.0], f)).tolist() == [0.0, np.inf, 0.0]
    assert O.qpu_exp(np.array([128.0], f), base2=True)[0] == np.inf


def test_division_within_four_ulp():
    rng = np.random.default_rng(1)
    a = rng.uniform(-10, 10, 10000).astype(f)
    b = rng.uniform(0.01, 100, 10000).astype(f)
    q = O.qpu_binary("fdiv", a, b)
    exact = a.astype(np.float64) / b.astype(np.float64)
    ulp = np.spacing(np.abs(exact).astype(f)).astype(np.float64)
    assert (np.abs(q - exact) / ulp).max() < 4.0      # Newton reciprocal, then a truncating multiply
    assert np.isnan(O.qpu_binary("fdiv", np.array([0.0], f), np.array([0.0], f))[0])


def test_softmax_rows_sum_to_one_and_masks():
    from piton_b200 import workloads as W
    x = W.softmax_input(16, 300, seed=5)
    y = O.qpu_softmax(x)
    assert np.all(y[np.isneginf(x)] == 0)
    np.testing.assert_allclose(y.sum(1), 1, atol=1e-5)
    np.testing.assert_allclose(y, O.softmax_f64(x), rtol=1e-5, atol=1e-12)


def test_attention_oracle_close_to_float64():
    from piton_b200 import workloads as W
    q, k, v = W.attention_inputs(2, 40, 16, seed=3)
    for causal in (False, True):
        o = O.qpu_attention(q, k, v, causal, 2, 16)
        np.testing.assert_allclose(o, O.attention_f64(q, k, v, causal), rtol=0, atol=2e-5)
