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
