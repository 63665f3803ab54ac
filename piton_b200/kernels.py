"""Declarations of the PIton example operators that run on the B200 backend.

Each function here has the parameter list of the reference's Triton source
(the launch interface) and a docstring saying what it computes; the body is
never executed.  ``kernel[grid](..., device="b200")`` binds the arguments as
the reference launcher does and runs the matching hand-written sm_100a kernel
(``piton_b200/csrc``).  The reference's own ``@piton.jit`` functions of the
same name and parameters are accepted too (the registry keys on the name and
parameter list), so a module written for PIton runs unchanged.
"""

from __future__ import annotations

from . import language as tl
from .jit import jit


@jit
def add_kernel(x_ptr, y_ptr, output_ptr, n_elements, BLOCK_SIZE: tl.constexpr):
    """output[i] = x[i] + y[i] for i < n_elements; program p owns
    [p*BLOCK_SIZE, (p+1)*BLOCK_SIZE).  (examples/kernels.py:6-15)"""


@jit
def matmul_kernel(a_ptr, b_ptr, c_ptr, M, N, K, stride_am, stride_ak, stride_bk, stride_bn, stride_cm, stride_cn,
                  BLOCK_SIZE_M: tl.constexpr, BLOCK_SIZE_N: tl.constexpr, BLOCK_SIZE_K: tl.constexpr,
                  GROUP_SIZE_M: tl.constexpr):
    """C = A @ B with element strides; program pid computes the C tile of the
    grouped (GROUP_SIZE_M) order; rows/cols past M/N are not stored.
    (examples/kernels.py:18-57)"""


@jit
def softmax_kernel(output_ptr, input_ptr, input_row_stride, output_row_stride, n_cols, BLOCK_SIZE: tl.constexpr):
    """Row softmax over the first min(n_cols, BLOCK_SIZE) columns; program p owns
    row p.  (examples/kernels.py:60-76)"""


@jit
def dense_layer_kernel(x_ptr, w_ptr, bias_ptr, y_ptr, M, N: tl.constexpr, K: tl.constexpr,
                       BLOCK_SIZE_M: tl.constexpr, BLOCK_SIZE_N: tl.constexpr, BLOCK_SIZE_K: tl.constexpr,
                       GROUP_SIZE_M: tl.constexpr, ADD_BIAS: tl.constexpr, RELU: tl.constexpr):
    """Y[M,N] = X[M,K] @ W[K,N] (+ bias) (ReLU), contiguous row-major.
    (examples/nn_kernels.py:23-74)"""


@jit
def attn_fwd_kernel(Q, K, V, Out, sm_scale, stride_qh, stride_qm, stride_kh, stride_kn, stride_kk, stride_vh,
                    stride_vn, stride_oh, stride_om, N_CTX, HEAD_DIM: tl.constexpr, BLOCK_M: tl.constexpr,
                    BLOCK_N: tl.constexpr, CAUSAL: tl.constexpr, EVEN_N: tl.constexpr):
    """Out = softmax(Q K^T * sm_scale) V per head (grid axis 1), causal or not.
    (examples/attention.py:75-113)"""


@jit
def layernorm_kernel(x_ptr, out_ptr, n, eps, BLOCK: tl.constexpr):
    """Row p: (x - mean) / sqrt(var + eps) over the first n of BLOCK columns,
    rows BLOCK apart.  (tests/test_reroll_reduce.py:199-208)"""


def dense_tiles(output_features):
    """(BM, BN, BK) the reference launches the digits layers with
    (examples/nn_kernels.py:14-20); on B200 they only decide grid coverage."""
    return (4, 64, 4) if output_features >= 64 else (8, 16, 4)


# ---- the other example / primitive operators (examples/primitive_kernels.py, elementwise.py,
# ---- sfu_tests.py, kernels.py:79-96, life.py)

@jit
def copy_kernel(x_ptr, out_ptr, n, BLOCK: tl.constexpr):
    """out[i] = x[i], i < n.  (examples/primitive_kernels.py:12-17)"""


@jit
def mul_kernel(x_ptr, y_ptr, out_ptr, n, BLOCK: tl.constexpr):
    """out[i] = x[i] * y[i].  (examples/elementwise.py:5-9)"""


@jit
def fma_kernel(x_ptr, y_ptr, out_ptr, n, alpha, BLOCK: tl.constexpr):
    """out[i] = x[i] * alpha + y[i] (multiply, then add).  (examples/primitive_kernels.py:20-27)"""


@jit
def scaled_relu_kernel(x_ptr, out_ptr, n, alpha, BLOCK: tl.constexpr):
    """out[i] = x[i] * alpha where x[i] > 0, else 0.  (examples/kernels.py:79-85)"""


@jit
def sfu_kernel(x_ptr, out_ptr, n, OP: tl.constexpr, BLOCK: tl.constexpr):
    """OP 0 exp2, 1 log2, 2 1/x, 3 rsqrt, 4 exp, 5 sqrt.  (examples/sfu_tests.py:5-21)"""


@jit
def log_kernel(x_ptr, out_ptr, n, BLOCK: tl.constexpr):
    """Natural log.  (examples/primitive_kernels.py:69-76)"""


@jit
def sigmoid_kernel(x_ptr, out_ptr, n, BLOCK: tl.constexpr):
    """out[i] = tl.sigmoid(x[i]) = 1 / (1 + exp(-x[i])), the language builtin applied element-wise
    (piton/language/core.py:787-790); the reference has no example kernel for it."""


@jit
def idiv_kernel(x_ptr, y_ptr, q_ptr, r_ptr, n, BLOCK: tl.constexpr):
    """Exact 32-bit x // y and x % y, C truncation (int32 or uint32 arrays).
    (examples/primitive_kernels.py:30-38)"""


@jit
def row_sum_kernel(x_ptr, out_ptr, n_cols, stride, BLOCK_M: tl.constexpr, BLOCK_N: tl.constexpr):
    """out[r] = sum of row r over ceil(n_cols / BLOCK_N) * BLOCK_N columns.  (examples/kernels.py:88-96)"""


@jit
def row_max_kernel(x_ptr, out_ptr, n_cols, stride, BLOCK_M: tl.constexpr, BLOCK_N: tl.constexpr):
    """out[r] = max of row r (from -FLT_MAX).  (examples/primitive_kernels.py:41-50)"""


@jit
def transpose_kernel(x_ptr, out_ptr, n_rows, n_cols, stride_x, stride_out, BLOCK_M: tl.constexpr,
                     BLOCK_N: tl.constexpr):
    """out[c, r] = x[r, c] per BLOCK_M x BLOCK_N tile.  (examples/primitive_kernels.py:53-66)"""


@jit
def life_kernel(src_ptr, dst_ptr, n_rows, n_cols, stride, BLOCK_R: tl.constexpr, BLOCK_C: tl.constexpr):
    """One Game of Life generation on a torus, int32 0/1 cells, tiles.  (examples/life.py:39-70)"""


@jit
def life_rows_kernel(src_ptr, dst_ptr, n_rows, n_cols, stride, ROWS: tl.constexpr, BLOCK: tl.constexpr):
    """The same generation, column strips walking rows.  (examples/life.py:73-101)"""


@jit
def life_bits_kernel(src_ptr, dst_ptr, n_rows, n_words, stride, ROWS: tl.constexpr, BLOCK: tl.constexpr):
    """The same generation on 32 cells per uint32 word.  (examples/life.py:113-147)"""
