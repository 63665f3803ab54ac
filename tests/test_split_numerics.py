"""The operand splits of the tensor-core GEMM and attention, modelled in numpy (no GPU).

GEMM (csrc/gemm_tc.cu): every 256-deep chunk of a row of A / column of B is scaled by a power
of two bringing its largest finite magnitude into [2^14, 2^15), split into fp16 halves
hi = fp16(s), lo = fp16(s - hi), and C = sum over chunks of 2^-(eA + eB) (A_hi B_hi + A_hi B_lo
+ A_lo B_hi).  Attention (csrc/attention_tc.cu): X_hi = X with the low 13 mantissa bits
cleared (a tf32 value), X_lo = X - X_hi (exact), and S = Q_hi K_hi + Q_hi K_lo (tf32) + one
bf16 product for the remaining cross term; the model of that tf32 + bf16 split below is the
GEMM's earlier scheme: C = A_hi B_hi + (A_lo B + A B_lo) with per group of 8 k-values the A
operand [bf16(A_lo), bf16(A)] and the B operand [bf16(B), bf16(B_lo)].  The models round the
operands exactly as the split kernels do and sum in float64, so they isolate the operand
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


# ---- the GEMM's fp16 split with per-chunk power-of-two scaling ------------------------------

KC = 256


def chunk_exponent(m):
    """15 - E for m = f 2^E, f in [0.5, 1): m 2^e in [2^14, 2^15); 0 for m == 0; clamp +-112."""
    m = np.asarray(m, np.float64)
    _, E = np.frexp(np.where(m > 0, m, 1.0))
    return np.where(m > 0, np.clip(15 - E, -112, 112), 0).astype(np.int64)


def split16(x):
    """x [rows, K] (K-major): hi, lo fp16 [rows, chunks, KC] (zero padded) and exponents [rows, chunks]."""
    x = np.asarray(x, np.float32)
    rows, K = x.shape
    chunks = -(-K // KC)
    xp = np.zeros((rows, chunks * KC), np.float32)
    xp[:, :K] = x
    xc = xp.reshape(rows, chunks, KC)
    e = chunk_exponent(np.abs(np.where(np.isfinite(xc), xc, 0)).max(-1))
    s = (xc * np.exp2(e)[..., None].astype(np.float32)).astype(np.float32)
    hi = s.astype(np.float16)
    lo = (s - hi.astype(np.float32)).astype(np.float16)
    return hi, lo, e


def f16_gemm(a, b):
    ah, al, ea = split16(a)
    bh, bl, eb = split16(np.asarray(b, np.float32).T)
    out = np.zeros((a.shape[0], b.shape[1]))
    for c in range(ah.shape[1]):
        Ah, Al = ah[:, c].astype(np.float64), al[:, c].astype(np.float64)
        Bh, Bl = bh[:, c].astype(np.float64), bl[:, c].astype(np.float64)
        acc = Ah @ Bh.T + Ah @ Bl.T + Al @ Bh.T
        out += acc * np.exp2(-(ea[:, c][:, None] + eb[:, c][None, :]))
    return out


def test_fp16_split_per_product_error():
    """Per product the dropped A_lo B_lo and the rounding of the low halves stay below 2^-20
    of |a b| wherever the values are within 2^10 of their chunk's largest."""
    rng = np.random.default_rng(1)
    a = (rng.uniform(1, 2, (512, KC)) * 2.0 ** rng.integers(-10, 1, (512, KC))).astype(np.float32)
    b = (rng.uniform(1, 2, (512, KC)) * 2.0 ** rng.integers(-10, 1, (512, KC))).astype(np.float32)
    ah, al, ea = split16(a)
    bh, bl, eb = split16(b)
    prod = (ah.astype(np.float64) * bh + ah.astype(np.float64) * bl + al.astype(np.float64) * bh)[:, 0]
    exact = a.astype(np.float64) * b * np.exp2(ea + eb)
    rel = np.abs(prod - exact) / np.abs(exact)
    assert rel.max() <= 2.0 ** -20


@pytest.mark.parametrize("K", [1000, 8192])
def test_fp16_split_dots_below_fp32_level(K):
    rng = np.random.default_rng(K)
    a = rng.uniform(-1, 1, (48, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, 40)).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    err = np.abs(f16_gemm(a, b) - exact).max() / np.abs(exact).max()
    fp32 = np.abs((a @ b).astype(np.float64) - exact).max() / np.abs(exact).max()
    assert err <= 1e-7 * np.sqrt(K) and err < fp32


def test_fp16_split_wide_dynamic_range():
    """Rows and columns spread over 2^-60 .. 2^60 (far beyond fp16's range): the per-chunk scale
    keeps every output at fp32 level relative to its own row and column magnitudes."""
    rng = np.random.default_rng(7)
    ra = np.exp2(rng.integers(-60, 61, 32)).astype(np.float32)
    cb = np.exp2(rng.integers(-60, 61, 24)).astype(np.float32)
    a = (rng.uniform(-1, 1, (32, 700)) * ra[:, None]).astype(np.float32)
    b = (rng.uniform(-1, 1, (700, 24)) * cb[None, :]).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    scale = np.abs(a).max(1)[:, None].astype(np.float64) * np.abs(b).max(0)[None, :]
    assert np.all(np.abs(f16_gemm(a, b) - exact) / scale <= 1e-7 * np.sqrt(700))


def test_chunk_exponent_range():
    e = chunk_exponent(np.array([1.0, 2.0 ** 14, 2.0 ** 15 - 1, 3e38, 1e-40, 0.0]))
    assert list(e) == [14, 0, 0, -112, 112, 0]
    m = np.array([1.0, 1.5, 65000.0, 1e-3])
    s = m * np.exp2(chunk_exponent(m))
    assert np.all((s >= 2.0 ** 14) & (s < 2.0 ** 15))
