"""The fp16 operand split of the tensor-core GEMM and attention, modelled in numpy (no GPU).

GEMM (csrc/gemm_tc.cu): every 256-deep chunk of a row of A / column of B is scaled by a power
of two bringing its largest finite magnitude into [2^14, 2^15), split into fp16 halves
hi = fp16(s), lo = fp16(s - hi), and C = sum over chunks of 2^-(eA + eB) (A_hi B_hi + A_hi B_lo
+ A_lo B_hi).  Attention (csrc/attention_tc.cu): the same split of each Q row (its own scale),
of each 64-key block of K and V (one scale per block) and of P in [0, 1] (scaled by 2^14).  The
models round the operands exactly as the split kernels do and sum in float64, so they isolate
the operand rounding (the tensor core's accumulation is covered by the GPU tests against
float64).
"""

import numpy as np
import pytest


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


def test_attention_p_split():
    """P in [0, 1] scaled by 2^14 and split into fp16 halves: relative error below 2^-21 where
    both halves are normal fp16 numbers, and below 2^-38 absolute for the smallest p, whose low
    half falls into fp16's subnormals (a 4096-key row of them moves an output by < 2^-26)."""
    rng = np.random.default_rng(3)
    p = np.concatenate([rng.uniform(0, 1, 100000), np.exp2(-rng.uniform(0, 60, 100000)), [0.0, 1.0]])
    p = p.astype(np.float32)
    s = (p * np.float32(16384.0)).astype(np.float32)
    hi = s.astype(np.float16)
    lo = (s - hi.astype(np.float32)).astype(np.float16)
    back = (hi.astype(np.float64) + lo.astype(np.float64)) / 16384.0
    err = np.abs(back - p.astype(np.float64))
    assert np.all(err <= np.maximum(2.0 ** -21 * p, 2.0 ** -38))
