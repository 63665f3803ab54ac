"""ctypes wrapper of the CPU oracle (qpu_oracle.c).

TEST INFRASTRUCTURE: imported only by tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py, as the checker.  The B200 product
path (piton_b200) never imports it.

Every function takes and returns float32 numpy arrays and follows the
reference's algorithm for the operator (see qpu_oracle.c for the file:line of
each restated step).  ``build()`` compiles liboracle.so with gcc when it is
missing or older than its source.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "qpu_oracle.c")
LIB = os.path.join(HERE, "liboracle.so")

_F = C.POINTER(C.c_float)
_i64, _int, _cf32 = C.c_int64, C.c_int, C.c_float
_lib = None


def build() -> str:
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB)
        L.oracle_add.argtypes = [_F, _F, _F, _i64]
        L.oracle_matmul.argtypes = [_F, _F, _F] + [_i64] * 9 + [_int]
        L.oracle_dense.argtypes = [_F, _F, _F, _F, _i64, _i64, _i64, _int, _int, _int]
        L.oracle_softmax.argtypes = [_F, _F, _i64, _i64, _i64, _i64, _i64]
        L.oracle_attention.argtypes = [_F, _F, _F, _F] + [_i64] * 12 + [_cf32, _int, _int, _i64, _i64]
        for name in ("oracle_map_fadd", "oracle_map_fmul", "oracle_map_fdiv"):
            getattr(L, name).argtypes = [_F, _F, _F, _i64]
        L.oracle_map_exp.argtypes = [_F, _F, _i64, _int]
        for f in (L.oracle_add, L.oracle_matmul, L.oracle_dense, L.oracle_softmax, L.oracle_attention):
            f.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_F)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def qpu_add(x, y):
    x, y = _f32(x), _f32(y)
    out = np.empty_like(x)
    lib().oracle_add(_p(x), _p(y), _p(out), x.size)
    return out


def qpu_binary(op: str, a, b):
    a, b = _f32(a), _f32(b)
    out = np.empty_like(a)
    getattr(lib(), f"oracle_map_{op}")(_p(a), _p(b), _p(out), a.size)
    return out


def qpu_exp(x, base2=False):
    x = _f32(x)
    out = np.empty_like(x)
    lib().oracle_map_exp(_p(x), _p(out), x.size, int(base2))
    return out


def qpu_matmul(a, b, threads: int = 1):
    """matmul_kernel with a covering grid: sequential-k round-toward-zero dots."""
    a, b = _f32(a), _f32(b)
    M, K = a.shape
    N = b.shape[1]
    c = np.zeros((M, N), np.float32)
    lib().oracle_matmul(_p(a), _p(b), _p(c), M, N, K, K, 1, N, 1, N, 1, int(threads))
    return c


def qpu_dense(x, w, bias, add_bias=True, relu=True, threads: int = 1):
    x, w, bias = _f32(x), _f32(w), _f32(bias)
    M, K = x.shape
    N = w.shape[1]
    y = np.zeros((M, N), np.float32)
    lib().oracle_dense(_p(x), _p(w), _p(bias), _p(y), M, N, K, int(add_bias), int(relu), int(threads))
    return y


def qpu_mlp(images, model, threads: int = 1):
    """digits forward (examples/digits_model.py:120-134) as three emulated dense layers."""
    h = (np.asarray(images).astype(np.float32) / np.float32(16)).astype(np.float32) \
        if np.issubdtype(np.asarray(images).dtype, np.integer) else _f32(images)
    for layer in (1, 2, 3):
        h = qpu_dense(h, model[f"w{layer}"], model[f"b{layer}"], True, layer < 3, threads)
    return h


def qpu_softmax(x, block=None):
    x = _f32(x)
    rows, n = x.shape
    block = block or (1 << (n - 1).bit_length())
    out = np.zeros_like(x)
    lib().oracle_softmax(_p(x), _p(out), rows, n, block, n, n)
    return out


def qpu_attention(q, k, v, causal, block_m=2, block_n=16, sm_scale=None, even_n=None):
    """attn_fwd_kernel over [H, N, D] contiguous q, k, v (K stored [N, D])."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    squeeze = q.ndim == 2
    if squeeze:
        q, k, v = q[None], k[None], v[None]
    h, n, d = q.shape
    sm_scale = float(1.0 / np.sqrt(d)) if sm_scale is None else float(sm_scale)
    even_n = (n % block_n == 0) if even_n is None else bool(even_n)
    o = np.zeros_like(q)
    lib().oracle_attention(_p(q), _p(k), _p(v), _p(o), h, n, d, n * d, d, n * d, d, 1, n * d, d, n * d, d,
                           sm_scale, int(causal), int(even_n), block_m, block_n)
    return o[0] if squeeze else o


# float64 references (the reference's own numpy checks: examples/attention.py:180-192,
# examples/digits_reference.py:14-55)

def attention_f64(q, k, v, causal, sm_scale=None):
    q, k, v = (np.asarray(x, np.float64) for x in (q, k, v))
    sm_scale = 1.0 / np.sqrt(q.shape[-1]) if sm_scale is None else sm_scale
    s = np.einsum("...md,...nd->...mn", q, k) * sm_scale
    if causal:
        n = s.shape[-1]
        s = np.where(np.tril(np.ones((s.shape[-2], n), bool)), s, -np.inf)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return p @ v


def softmax_f64(x):
    x = np.asarray(x, np.float64)
    e = np.exp(x - x.max(axis=1, keepdims=True))
    return e / e.sum(axis=1, keepdims=True)


def mlp_f64_with_bounds(images, model):
    """float64 logits and per-logit round-toward-zero error bounds
    gamma = (2K+1) 2^-23 per layer, propagated through |W| (digits_reference.py:14-55)."""
    images = np.asarray(images)
    act = images.astype(np.float64) / 16.0 if np.issubdtype(images.dtype, np.integer) \
        else images.astype(np.float32).astype(np.float64)
    err = np.zeros_like(act)
    for layer, (k, n) in enumerate(((64, 128), (128, 64), (64, 16)), start=1):
        w = np.asarray(model[f"w{layer}"], np.float64)
        b = np.asarray(model[f"b{layer}"], np.float64)
        g = (2 * k + 1) * 2.0 ** -23
        g = g / (1 - g)
        err = (err @ np.abs(w)) * (1 + g) + g * (np.abs(act) @ np.abs(w) + np.abs(b))
        act = act @ w + b
        if layer < 3:
            act = np.maximum(act, 0.0)
    return act, err


# ---- integer division, Life, element-wise QPU ops -----------------------------------------

def idiv_c(x, y, signed=True):
    """C-semantics 32-bit // and % as uint32 bit patterns (INT_MIN / -1 wraps), the
    definition the reference checks its exact division against (tests/test_fast_idiv.py:146-155)."""
    M32 = 0xFFFFFFFF
    a = np.asarray(x).view(np.uint32)
    b = np.asarray(y).view(np.uint32)
    if signed:
        xa, yb = a.view(np.int32).astype(np.int64), b.view(np.int32).astype(np.int64)
        q = np.sign(xa) * np.sign(yb) * (np.abs(xa) // np.abs(yb))
        r = xa - q * yb
    else:
        xa, yb = a.astype(np.int64), b.astype(np.int64)
        q, r = xa // yb, xa % yb
    return (q & M32).astype(np.uint32), (r & M32).astype(np.uint32)


def life_step(cells):
    """One generation on a torus: alive next iff the 3x3 block (cell included) holds 3 live
    cells, or 4 and the cell is alive (examples/life.py:1-20)."""
    c = np.asarray(cells).astype(np.int64)
    t = sum(np.roll(np.roll(c, dr, 0), dc, 1) for dr in (-1, 0, 1) for dc in (-1, 0, 1))
    return ((t == 3) | ((t == 4) & (c != 0))).astype(np.int32)


def pack_bits(cells):
    """32 cells per uint32 word, bit j of word k = column 32k + j."""
    return np.packbits(np.asarray(cells, np.uint8), axis=1, bitorder="little").view(np.uint32)


def unpack_bits(words, n_cols):
    return np.unpackbits(np.ascontiguousarray(words).view(np.uint8), axis=1, bitorder="little")[:, :n_cols]


def qpu_fma(x, y, alpha):
    """x * alpha + y as two round-toward-zero operations (no fused multiply-add on the QPU)."""
    a = np.full(np.shape(x), np.float32(alpha), np.float32)
    return qpu_binary("fadd", qpu_binary("fmul", x, a), y)


def qpu_scaled_relu(x, alpha):
    x = _f32(x)
    p = qpu_binary("fmul", x, np.full(x.shape, np.float32(alpha), np.float32))
    return np.where(x > 0, p, np.float32(0)).astype(np.float32)
