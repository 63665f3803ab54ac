"""Empty and degenerate launches, as the reference's programs define them: a zero-sized
extent or an empty grid launches no work and leaves every output untouched; a matmul with
K = 0 runs no k-iteration, so its tiles store the zero accumulator (examples/kernels.py:
the K loop of matmul_kernel); the digits MLP and TinyGPT accept a batch of 0."""

import numpy as np
import pytest

import piton_b200 as triton
from piton_b200 import digits, tinygpt
from piton_b200 import workloads as W
from piton_b200.kernels import add_kernel, attn_fwd_kernel, matmul_kernel, softmax_kernel

pytestmark = pytest.mark.gpu


def test_add_with_no_elements_or_no_programs(cuda):
    x = np.ones(64, np.float32)
    out = np.full(64, 7.0, np.float32)
    add_kernel[(1,)](x, x, out, 0, BLOCK_SIZE=64, device="b200")       # one program, n = 0: all masked
    assert np.all(out == 7.0)
    add_kernel[(0,)](x, x, out, 64, BLOCK_SIZE=64, device="b200")      # no programs
    assert np.all(out == 7.0)


def test_softmax_with_no_rows_or_no_columns(cuda):
    x = np.random.default_rng(0).standard_normal((4, 64)).astype(np.float32)
    out = np.full((4, 64), 3.0, np.float32)
    softmax_kernel[(0,)](out, x, 64, 64, 64, BLOCK_SIZE=64, device="b200")
    assert np.all(out == 3.0)
    softmax_kernel[(4,)](out, x, 64, 64, 0, BLOCK_SIZE=64, device="b200")   # n_cols = 0: every column masked
    assert np.all(out == 3.0)


@pytest.mark.parametrize("M,N", [(0, 64), (64, 0)])
def test_matmul_with_an_empty_output(cuda, M, N):
    K = 32
    a = np.ones((max(M, 1), K), np.float32)
    b = np.ones((K, max(N, 1)), np.float32)
    c = np.full((max(M, 1), max(N, 1)), 5.0, np.float32)
    grid = (max(1, triton.cdiv(M, 8) * triton.cdiv(N, 64)),)
    matmul_kernel[grid](a, b, c, M, N, K, K, 1, max(N, 1), 1, max(N, 1), 1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64,
                        BLOCK_SIZE_K=8, GROUP_SIZE_M=8, device="b200")
    assert np.all(c == 5.0)


@pytest.mark.parametrize("M,N", [(64, 64), (512, 640)])
def test_matmul_with_k_zero_stores_zeros(cuda, M, N):
    a = np.ones((M, 1), np.float32)
    b = np.ones((1, N), np.float32)
    c = np.full((M, N), 5.0, np.float32)
    matmul_kernel[(triton.cdiv(M, 8) * triton.cdiv(N, 64),)](a, b, c, M, N, 0, 1, 1, N, 1, N, 1, BLOCK_SIZE_M=8,
                                                              BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8,
                                                              device="b200")
    assert np.all(c == 0.0)


def test_attention_with_no_query_rows(cuda):
    heads, n, d = 1, 64, 64
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((heads, n, d)).astype(np.float32) for _ in range(3))
    out = np.full_like(q, 2.0)
    attn_fwd_kernel[(0, heads)](q, k, v, out, 0.125, n * d, d, n * d, d, 1, n * d, d, n * d, d, n, HEAD_DIM=d,
                                BLOCK_M=2, BLOCK_N=16, CAUSAL=True, EVEN_N=True, device="b200")
    assert np.all(out == 2.0)


def test_mlp_and_tinygpt_with_a_batch_of_zero(cuda):
    torch = cuda
    model = digits.DigitsMLP(W.digits_model(0))
    x = torch.zeros(0, 64, dtype=torch.uint8, device="cuda")
    logits = torch.zeros(0, 16, device="cuda")
    model.forward_device(x, logits)
    gpt = tinygpt.TinyGPT(tinygpt.init_weights(0))
    toks = torch.zeros(0, tinygpt.CTX, dtype=torch.int32, device="cuda")
    gpt.generate_device(toks, 16, 8)
    torch.cuda.synchronize()
