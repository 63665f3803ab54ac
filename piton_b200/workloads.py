"""Seeded synthetic inputs for every operator on the hot path.

Each generator takes a seed and a size and returns float32 numpy arrays with
the shapes and value distributions the benchmark configurations name:

* vector add: x, y ~ U[-1, 1]                     (examples/kernels.py:6-15)
* fused softmax: N(0, 1) * 4 with 1% of every row set to -inf, at least one
  finite entry per row                            (examples/kernels.py:60-76)
* grouped matmul: A, B ~ U[-1, 1]                 (examples/kernels.py:18-57)
* causal attention: Q, K, V ~ N(0, 1), scale 1/sqrt(D)
                                                  (examples/attention.py:75-113)
* digits MLP: 8x8 images with integer intensities 0..16 and synthetic weights
  in the reference's model layout (w1 64x128, b1 128, w2 128x64, b2 64,
  w3 64x16, b3 16 with the six padding outputs zero; examples/digits_model.py:31-38)
* dyadic dense-layer inputs whose products and sums are exact in fp32
  (tests/test_nn_kernels.py:43-48 uses the same idea for a bit comparison)

The same generators feed the golden-fixture script, the parity tests and the
benchmark, so all three see identical inputs for a given seed.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def vector_add(n: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1.0, 1.0, n).astype(F32)
    y = rng.uniform(-1.0, 1.0, n).astype(F32)
    return x, y


def softmax_input(m: int, n: int, seed: int = 0, neg_inf_frac: float = 0.01):
    """N(0,1)*4 rows with round(frac*n) entries (at least one, at most n-1) set to -inf."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((m, n)) * 4.0).astype(F32)
    k = int(round(neg_inf_frac * n))
    k = max(1, min(k, n - 1)) if n > 1 else 0
    if k:
        # one permutation draw per row, vectorised: argsort of uniform keys
        cols = np.argsort(rng.random((m, n)), axis=1)[:, :k]
        np.put_along_axis(x, cols, -np.inf, axis=1)
    return x


def matmul_inputs(m: int, n: int, k: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    a = rng.uniform(-1.0, 1.0, (m, k)).astype(F32)
    b = rng.uniform(-1.0, 1.0, (k, n)).astype(F32)
    return a, b


def attention_inputs(bh: int, s: int, d: int, seed: int = 0, gain: float = 1.0):
    """Q, K, V as [B*H, S, D] contiguous fp32."""
    rng = np.random.default_rng(seed)
    q, k, v = (rng.standard_normal((bh, s, d)).astype(F32) for _ in range(3))
    if gain != 1.0:
        q = (q * F32(gain)).astype(F32)
    return q, k, v


def digits_images(n: int, seed: int = 0):
    """n synthetic 8x8 images, integer intensities 0..16 (uint8, shape (n, 64))."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, 17, (n, 64)).astype(np.uint8)


def digits_model(seed: int = 0):
    """Synthetic weights in the digits model layout; the last six outputs are zero padding."""
    rng = np.random.default_rng(seed)
    model = {}
    for layer, (k, n) in enumerate(((64, 128), (128, 64), (64, 16)), start=1):
        w = rng.normal(0.0, 1.0 / np.sqrt(k), (k, n)).astype(F32)
        b = rng.normal(0.0, 0.05, n).astype(F32)
        model[f"w{layer}"] = w
        model[f"b{layer}"] = b
    model["w3"][:, 10:] = 0
    model["b3"][10:] = 0
    return model


def dyadic(shape, lo: int, hi: int, rng: np.random.Generator, denom: float = 4.0):
    return (rng.integers(lo, hi + 1, shape).astype(F32) / F32(denom)).astype(F32)
