"""Causal / full attention on the B200 (examples/attention.py:33-113).

Mirrors tests/test_attention.py of the reference: ATOL 2e-5 against float64
and against the oracle (bit-exact with the emulator goldens), ragged N_CTX
with sentinel rows past the end, multi-head runtime strides through the
launcher, transposed K, hard attention, causal rows independent of future keys.
"""

import numpy as np
import pytest

from conftest import golden_ids, goldens, sha256
from oracle import oracle as O
from piton_b200 import workloads as W
from piton_b200.kernels import attn_fwd_kernel

pytestmark = pytest.mark.gpu
ATTN = goldens("attn_")
ATOL = 2e-5


def qkv(n, d, seed=0, gain=1.0, heads=None):
    rng = np.random.default_rng(seed)
    shape = (n, d) if heads is None else (heads, n, d)
    q, k, v = (rng.standard_normal(shape).astype(np.float32) for _ in range(3))
    return (q * np.float32(gain)).astype(np.float32), k, v


def run(q, k, v, causal, block_m=2, block_n=16, k_layout="nd", out=None, even_n=None, qpu=False):
    squeeze = q.ndim == 2
    if squeeze:
        q, k, v = q[None], k[None], v[None]
    h, n, d = q.shape
    kk = np.ascontiguousarray(k.transpose(0, 2, 1)) if k_layout == "dn" else k
    s_kn, s_kk = (1, n) if k_layout == "dn" else (d, 1)
    o = np.zeros_like(q) if out is None else out
    even = (n % block_n == 0) if even_n is None else even_n
    grid = (-(-n // block_m), h)
    attn_fwd_kernel[grid](q, kk, v, o, float(1 / np.sqrt(d)), n * d, d, n * d, s_kn, s_kk, n * d, d,
                          o.shape[-2] * d if o.ndim == 3 else 0, d, n, HEAD_DIM=d, BLOCK_M=block_m,
                          BLOCK_N=block_n, CAUSAL=bool(causal), EVEN_N=bool(even), device="b200",
                          **({"qpu_rounding": True} if qpu else {}))
    return o[0] if squeeze else o


@pytest.mark.parametrize("n,d,block_m,block_n,causal", [
    (64, 16, 2, 16, False), (64, 16, 2, 16, True), (64, 32, 2, 32, False), (64, 32, 2, 32, True),
    (64, 32, 4, 16, False), (32, 64, 2, 16, True), (256, 128, 2, 16, True)])
def test_matches_float64(cuda, n, d, block_m, block_n, causal):
    q, k, v = qkv(n, d, seed=n + d + block_m)
    out = run(q, k, v, causal, block_m, block_n)
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, O.attention_f64(q, k, v, causal), rtol=0, atol=ATOL)


@pytest.mark.parametrize("g", ATTN, ids=golden_ids(ATTN))
def test_matches_emulator_golden(cuda, g):
    m = g.meta
    q, k, v = W.attention_inputs(m["heads"], m["n"], m["d"], m["seed"])
    out = run(q, k, v, m["causal"], m["block"][0], m["block"][1])
    ref = O.qpu_attention(q, k, v, m["causal"], m["block"][0], m["block"][1])
    np.testing.assert_allclose(out, ref, rtol=0, atol=ATOL)


@pytest.mark.parametrize("g", ATTN, ids=golden_ids(ATTN))
def test_qpu_rounding_bit_exact_with_emulator(cuda, g):
    """qpu_rounding=True: the reference program on the QPU float model, every output word equal to
    the emulator's (the fixture holds the SHA-256 of its whole output)."""
    m = g.meta
    q, k, v = W.attention_inputs(m["heads"], m["n"], m["d"], m["seed"])
    out = run(q, k, v, m["causal"], m["block"][0], m["block"][1], qpu=True)
    assert sha256(out) == m["sha_out"]


@pytest.mark.parametrize("n,d,block_m,block_n,causal,even", [
    (37, 16, 2, 16, True, False), (37, 16, 4, 16, False, False), (64, 32, 2, 32, False, True),
    (100, 64, 8, 64, True, False), (130, 128, 2, 128, False, False), (48, 16, 3, 8, True, True)])
def test_qpu_rounding_matches_oracle(cuda, n, d, block_m, block_n, causal, even):
    """Ragged contexts, BLOCK_N from 8 to 128, BLOCK_M not a divisor, EVEN_N both ways: bit for bit
    with the oracle's restatement (which matches the emulator goldens)."""
    q, k, v = qkv(n, d, seed=n * d + block_n)
    if even and n % block_n:
        pytest.skip("EVEN_N promises N_CTX % BLOCK_N == 0")
    out = run(q, k, v, causal, block_m, block_n, even_n=even, qpu=True)
    ref = O.qpu_attention(q, k, v, causal, block_m, block_n, even_n=even)
    np.testing.assert_array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_config_b4_h4_s256_d64(cuda):
    q, k, v = W.attention_inputs(16, 256, 64, 0)
    out = run(q, k, v, True)
    np.testing.assert_allclose(out, O.qpu_attention(q, k, v, True), rtol=0, atol=ATOL)
    np.testing.assert_allclose(out, O.attention_f64(q, k, v, True), rtol=0, atol=ATOL)


@pytest.mark.parametrize("n,causal", [(37, False), (37, True), (1, False), (17, True), (200, True)])
def test_ragged_sequence_lengths(cuda, n, causal):
    q, k, v = qkv(n, 16, seed=n)
    sentinel = np.float32(-1234.5)
    out = np.full((1, n + 3, 16), sentinel, np.float32)
    run(q[None], k[None], v[None], causal, 2, 16, out=out)
    np.testing.assert_array_equal(out[0, n:], sentinel)
    np.testing.assert_allclose(out[0, :n], O.attention_f64(q, k, v, causal), rtol=0, atol=ATOL)
    if n == 1:
        np.testing.assert_array_max_ulp(out[0, :1], v, maxulp=2)


def test_multi_head_runtime_strides_through_the_launcher(cuda):
    heads, n, d, pad = 2, 48, 16, 8
    rng = np.random.default_rng(5)
    q_store = rng.standard_normal((heads, n, d + pad)).astype(np.float32)
    k, v = (rng.standard_normal((heads, n, d)).astype(np.float32) for _ in range(2))
    out = np.zeros((heads, n, d), np.float32)
    attn_fwd_kernel[(n // 2, heads)](q_store, k, v, out, float(1 / np.sqrt(d)), n * (d + pad), d + pad, n * d, d, 1,
                                     n * d, d, n * d, d, n, HEAD_DIM=d, BLOCK_M=2, BLOCK_N=16, CAUSAL=True,
                                     EVEN_N=True, device="b200")
    ref = O.attention_f64(q_store[:, :, :d], k, v, causal=True)
    np.testing.assert_allclose(out, ref, rtol=0, atol=ATOL)


def test_transposed_k_layout_is_bit_identical(cuda):
    q, k, v = qkv(32, 32, seed=11)
    nd = run(q, k, v, False, 2, 16, k_layout="nd")
    dn = run(q, k, v, False, 2, 16, k_layout="dn")
    np.testing.assert_array_equal(nd.view(np.uint32), dn.view(np.uint32))


def test_hard_attention_retrieves_values(cuda):
    n = d = 32
    rng = np.random.default_rng(3)
    perm = rng.permutation(n)
    k = np.eye(n, dtype=np.float32)
    q = (1000.0 * np.eye(n, dtype=np.float32)[perm]).astype(np.float32)
    v = rng.standard_normal((n, d)).astype(np.float32)
    out = run(q, k, v, False, 2, 16)
    np.testing.assert_array_max_ulp(out, v[perm], maxulp=2)


def test_causal_rows_ignore_future_keys(cuda):
    n, d = 48, 16
    q, k, v = qkv(n, d, seed=8)
    a = run(q, k, v, True)
    k2, v2 = k.copy(), v.copy()
    rng = np.random.default_rng(9)
    k2[32:] = rng.standard_normal((n - 32, d)) * 10
    v2[32:] = rng.standard_normal((n - 32, d)) * 10
    b = run(q, k2, v2, True)
    np.testing.assert_array_equal(a[:32].view(np.uint32), b[:32].view(np.uint32))
    np.testing.assert_array_max_ulp(a[0], v[0], maxulp=2)
    assert not np.array_equal(a[32:], b[32:])


def test_large_scores_stay_finite(cuda):
    q, k, v = qkv(48, 16, seed=4, gain=25.0)
    out = run(q, k, v, False)
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, O.attention_f64(q, k, v, False), rtol=0, atol=ATOL)


def test_even_n_promise_skips_ragged_tail_like_the_reference(cuda):
    # EVEN_N=True on a non-causal launch with N_CTX % BLOCK_N != 0: the reference
    # skips the last partial key block (examples/attention.py:104-111)
    q, k, v = qkv(40, 16, seed=2)
    out = run(q, k, v, False, 2, 16, even_n=True)
    np.testing.assert_allclose(out, O.qpu_attention(q, k, v, False, 2, 16, even_n=True), rtol=0, atol=ATOL)


def _status():
    import ctypes
    from piton_b200.runtime.cuda._lib import lib
    st = ctypes.c_int(-1)
    assert lib().piton_b200_device_status(ctypes.byref(st)) == 0
    return st.value


@pytest.mark.parametrize("heads,n,causal", [(1, 64, True), (2, 100, False), (3, 200, True), (1, 1000, True),
                                            (2, 513, False), (1, 64, False)])
def test_tensor_core_path(cuda, monkeypatch, heads, n, causal):
    q, k, v = qkv(n, 64, seed=heads * n, heads=heads)
    sentinel = np.float32(-1234.5)
    out = np.full((heads, n + 2, 64), sentinel, np.float32)
    h, _, d = q.shape
    stats = attn_fwd_kernel[(-(-n // 2), h)](q, k, v, out, float(1 / np.sqrt(d)), n * d, d, n * d, d, 1, n * d, d,
                                              (n + 2) * d, d, n, HEAD_DIM=d, BLOCK_M=2, BLOCK_N=16,
                                              CAUSAL=causal, EVEN_N=n % 16 == 0, device="b200").last_stats
    assert stats["path"] == "tcgen05_f16x3"
    assert _status() == 0
    np.testing.assert_array_equal(out[:, n:], sentinel)
    np.testing.assert_allclose(out[:, :n], O.attention_f64(q, k, v, causal), rtol=0, atol=ATOL)
    monkeypatch.setenv("PITON_B200_FORCE_SIMT", "1")
    simt = run(q, k, v, causal, 2, 16)
    np.testing.assert_allclose(out[:, :n], simt, rtol=0, atol=ATOL)


def test_tensor_core_path_strided_k_and_padded_rows(cuda):
    # K pre-transposed [D, N] and Q / Out rows padded to 80 floats
    heads, n, d = 2, 192, 64
    rng = np.random.default_rng(17)
    q = rng.standard_normal((heads, n, 80)).astype(np.float32)
    k, v = (rng.standard_normal((heads, n, d)).astype(np.float32) for _ in range(2))
    kt = np.ascontiguousarray(k.transpose(0, 2, 1))
    out = np.zeros((heads, n, 80), np.float32)
    stats = attn_fwd_kernel[(n // 2, heads)](q, kt, v, out, 0.125, n * 80, 80, n * d, 1, n, n * d, d, n * 80, 80, n,
                                             HEAD_DIM=d, BLOCK_M=2, BLOCK_N=16, CAUSAL=True, EVEN_N=True,
                                             device="b200").last_stats
    assert stats["path"] == "tcgen05_f16x3"
    np.testing.assert_allclose(out[:, :, :d], O.attention_f64(q[:, :, :d], k, v, True), rtol=0, atol=ATOL)
    assert np.all(out[:, :, d:] == 0)


@pytest.mark.parametrize("q_off", [0, 1])
def test_tensor_core_path_unaligned_q_and_out(cuda, q_off):
    """Q rows 65 floats apart (and, with q_off = 1, a Q base off the 16-byte grid) cannot be
    read by TMA in place: the kernel works from a contiguous copy of Q; Out rows 65 apart take
    the scalar stores."""
    from piton_b200.runtime.launcher import offset_ptr
    heads, n, d, ld = 2, 256, 64, 65
    rng = np.random.default_rng(23 + q_off)
    qbuf = rng.standard_normal(heads * n * ld + 8).astype(np.float32)
    q = qbuf[q_off:q_off + heads * n * ld].reshape(heads, n, ld)
    k, v = (rng.standard_normal((heads, n, d)).astype(np.float32) for _ in range(2))
    out = np.full((heads, n, ld), 3.0, np.float32)
    stats = attn_fwd_kernel[(n // 2, heads)](offset_ptr(qbuf, q_off), k, v, out, 0.125, n * ld, ld, n * d, d, 1,
                                             n * d, d, n * ld, ld, n, HEAD_DIM=d, BLOCK_M=2, BLOCK_N=16,
                                             CAUSAL=False, EVEN_N=True, device="b200").last_stats
    assert stats["path"] == "tcgen05_f16x3"
    assert _status() == 0
    np.testing.assert_allclose(out[:, :, :d], O.attention_f64(q[:, :, :d], k, v, False), rtol=0, atol=ATOL)
    assert np.all(out[:, :, d:] == 3.0)


@pytest.mark.parametrize("k_ld,k_gap,v_ld", [(68, 0, 68), (65, 0, 65), (64, 4, 64), (64, 0, 72)])
def test_tensor_core_path_k_and_v_layouts(cuda, k_ld, k_gap, v_ld):
    """K rows k_ld floats apart with k_gap extra floats between heads, V rows v_ld apart: K read in
    place as its own high half (rows one stride apart across heads, 16-byte multiples), the
    vectorised K split (16-byte rows, heads not one stride apart), or the strided one (odd row
    stride); V through the 64 x 64-tile transposing split (16-byte rows) or the strided one."""
    heads, n, d = 2, 200, 64
    rng = np.random.default_rng(k_ld + 10 * k_gap + v_ld)
    q = rng.standard_normal((heads, n, d)).astype(np.float32)
    k = rng.standard_normal((heads, n, d)).astype(np.float32)
    v = rng.standard_normal((heads, n, d)).astype(np.float32)
    skh, svh = n * k_ld + k_gap, n * v_ld
    kbuf = np.full(heads * skh, np.nan, np.float32)
    vbuf = np.full(heads * svh, np.nan, np.float32)
    for h in range(heads):
        kbuf[h * skh:h * skh + n * k_ld].reshape(n, k_ld)[:, :d] = k[h]
        vbuf[h * svh:h * svh + n * v_ld].reshape(n, v_ld)[:, :d] = v[h]
    out = np.zeros_like(q)
    stats = attn_fwd_kernel[(n // 2, heads)](q, kbuf, vbuf, out, 0.125, n * d, d, skh, k_ld, 1, svh, v_ld, n * d, d, n,
                                             HEAD_DIM=d, BLOCK_M=2, BLOCK_N=8, CAUSAL=True, EVEN_N=True,
                                             device="b200").last_stats
    assert stats["path"] == "tcgen05_f16x3"
    assert _status() == 0
    np.testing.assert_allclose(out, O.attention_f64(q, k, v, True), rtol=0, atol=ATOL)
