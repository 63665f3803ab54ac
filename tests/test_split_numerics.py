"""The operand split of the tensor-core GEMM and attention, modelled in numpy (no GPU).

The kernels compute C = A_hi B_hi + (A_lo B + A B_lo) with A_hi = A with the low 13
mantissa bits cleared (a tf32 value), A_lo = A - A_hi (exact), the first product in tf32
(exact products) and the bracket as one bf16 product: per group of 8 k-values the A operand
holds [bf16(A_lo), bf16(A)] and the B operand [bf16(B), bf16(B_lo)].  The model rounds the
operands exactly as the split kernels do and sums in float64, so it isolates the operand
rounding (the tensor core's accumulation is covered by the GPU tests against float64).

Checked: the rounding error per product is at most 2^-17 + 2^-20 of |a b| (each cross term is
within 2^-8 of a term at most 2^-10 of the product, and A_lo B_lo <= 2^-20 is counted twice),
below 2^-19 rms and unbiased (the classic three-term tf32 split: below 2^-19 worst case); dot
products of the benchmark's depth stay at the fp32 level (far below the 2e-5 * sqrt(K)
contract); non-finite operands contribute nothing to the bracket.
"""

import numpy as np
import pytest


def tf32_hi(x):
    return (np.asarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


def bf16(x):
    """Round-to-nearest-even to bf16 (non-finite -> 0 and clamping as the split kernels do)."""
    x = np.asarray(x, np.float32)
    big = np.float32(3.3895313892515355e38)
    x = np.where(np.isfinite(x), np.clip(x, -big, big), np.float32(0)).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return u.astype(np.uint32).view(np.float32)


def split_product(a, b):
    """Elementwise model of one k-term: hi*hi + (lo_a * b + a * lo_b), in float64."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    ah, bh = tf32_hi(a), tf32_hi(b)
    with np.errstate(invalid="ignore"):
        al = np.where(np.isfinite(a), a - ah, 0).astype(np.float32)
        bl = np.where(np.isfinite(b), b - bh, 0).astype(np.float32)
    cross = bf16(al).astype(np.float64) * bf16(b) + bf16(a).astype(np.float64) * bf16(bl)
    return ah.astype(np.float64) * bh + cross


def three_tf32_product(a, b):
    """The classic 3xTF32 split: hi*hi + hi*lo + lo*hi with lo = tf32(x - hi)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    ah, bh = tf32_hi(a), tf32_hi(b)
    al, bl = tf32_hi(a - ah), tf32_hi(b - bh)
    return ah.astype(np.float64) * bh + ah.astype(np.float64) * bl + al.astype(np.float64) * bh


def test_bf16_rounding_matches_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, 1.0078125, -2.5, 3.0e38, 1e-30], np.float32)
    got = bf16(x)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: even mantissa -> 1
    assert got[1] == np.float32(1.0)
    assert got[2] == np.float32(1.0078125)
    assert got[4] == np.float32(-2.5)
    assert np.isfinite(got[5])
    assert np.all(np.abs(got - x) <= np.abs(x) * 2.0 ** -8)


def test_per_product_error_bound_and_bias():
    rng = np.random.default_rng(0)
    # values across the full mantissa range and several binades
    a = (rng.uniform(1, 2, 200000) * 2.0 ** rng.integers(-8, 8, 200000) * rng.choice([-1, 1], 200000)).astype(np.float32)
    b = (rng.uniform(1, 2, 200000) * 2.0 ** rng.integers(-8, 8, 200000) * rng.choice([-1, 1], 200000)).astype(np.float32)
    exact = a.astype(np.float64) * b
    rel = (split_product(a, b) - exact) / np.abs(exact)
    assert np.abs(rel).max() <= 2.0 ** -17 + 2.0 ** -20
    assert rel.std() < 2.0 ** -19
    # unbiased: the mean signed error is far below its spread
    assert abs(rel.mean()) < 0.02 * rel.std()
    # the three-term tf32 split for comparison
    rel3 = (three_tf32_product(a, b) - exact) / np.abs(exact)
    assert np.abs(rel3).max() < 2.0 ** -19


@pytest.mark.parametrize("K", [1024, 8192])
def test_dot_products_at_fp32_level(K):
    rng = np.random.default_rng(K)
    M = N = 48
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    model = np.einsum("mk,kn->mn", np.zeros((M, K)), np.zeros((K, N)))
    for k0 in range(0, K, 256):
        sl = slice(k0, k0 + 256)
        model += split_product(a[:, sl, None], b[None, sl, :]).sum(axis=1)
    err = np.abs(model - exact).max() / np.abs(exact).max()
    assert err <= 1e-7 * np.sqrt(K)                 # fp32 level; the contract is 2e-5 * sqrt(K)
    fp32 = (a @ b).astype(np.float64)               # numpy's fp32 GEMM for scale
    assert err <= 4 * np.abs(fp32 - exact).max() / np.abs(exact).max() + 1e-9


def test_non_finite_operands_leave_the_cross_terms_out():
    a = np.array([np.inf, -np.inf, np.nan, 1.5], np.float32)
    b = np.array([2.0, 0.75, 1.0, np.inf], np.float32)
    ah, bh = tf32_hi(a), tf32_hi(b)
    with np.errstate(invalid="ignore"):
        al = np.where(np.isfinite(a), a - ah, 0).astype(np.float32)
        bl = np.where(np.isfinite(b), b - bh, 0).astype(np.float32)
    cross = bf16(al).astype(np.float64) * bf16(b) + bf16(a).astype(np.float64) * bf16(bl)
    assert np.all(cross[:3] == 0) and cross[3] == 0
    # so the product is the tf32 one: inf * 2 = inf, -inf * 0.75 = -inf, nan stays nan
    prod = ah.astype(np.float64) * bh + cross
    assert prod[0] == np.inf and prod[1] == -np.inf and np.isnan(prod[2]) and prod[3] == np.inf
