"""The launch surface without a GPU: binding rules (piton/runtime/launcher.py:25-63),
device dispatch (:238-244), the registry, the accessed-extent checks and the
reference's own JITFunction objects (when PITON_REFERENCE names a reference checkout)."""

import os
import sys

import numpy as np
import pytest

import piton_b200 as triton
from piton_b200 import language as tl
from piton_b200.kernels import add_kernel, attn_fwd_kernel, dense_layer_kernel, matmul_kernel, softmax_kernel
from piton_b200.runtime import cuda
from piton_b200.runtime.launcher import bind, offset_ptr, parse_device


def test_cdiv_and_next_power_of_2():
    assert triton.cdiv(65537, 256) == 257
    assert triton.next_power_of_2(781) == 1024 and triton.next_power_of_2(1) == 1


def test_direct_call_raises():
    with pytest.raises(RuntimeError):
        add_kernel(1, 2, 3, 4)


def test_bind_specialises_constexprs_and_ones():
    x = np.zeros(4, np.float32)
    sig, consts, vals = bind(matmul_kernel.fn, (x, x, x, 4, 4, 4, 4, 1, 4, 1, 4, 1),
                             dict(BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8, GROUP_SIZE_M=8))
    assert consts == dict(stride_ak=1, stride_bn=1, stride_cn=1, BLOCK_SIZE_M=8, BLOCK_SIZE_N=64, BLOCK_SIZE_K=8,
                          GROUP_SIZE_M=8)
    assert sig["a_ptr"] == "*fp32" and sig["M"] == "i32"
    assert set(vals) == {"a_ptr", "b_ptr", "c_ptr", "M", "N", "K", "stride_am", "stride_bk", "stride_cm"}


def test_bind_rejects_unsupported_dtypes_and_missing_args():
    with pytest.raises(TypeError):
        bind(add_kernel.fn, (np.zeros(4, np.float64), np.zeros(4, np.float32), np.zeros(4, np.float32), 4),
             dict(BLOCK_SIZE=4))
    with pytest.raises(TypeError):
        bind(add_kernel.fn, (np.zeros(4, np.float32),), dict(BLOCK_SIZE=4))
    sig, _, _ = bind(add_kernel.fn, (offset_ptr(np.zeros(4, np.int32), 2), np.zeros(4, np.uint32),
                                     np.zeros(4, np.float32), 2.5), dict(BLOCK_SIZE=4))
    assert sig == {"x_ptr": "*i32", "y_ptr": "*u32", "output_ptr": "*fp32", "n_elements": "fp32"}


def test_unknown_device_is_a_value_error():
    x = np.zeros(4, np.float32)
    for dev in ("emu", "pi", "cuda", "b100"):
        with pytest.raises(ValueError):
            add_kernel[(1,)](x, x, x, 4, BLOCK_SIZE=4, device=dev)
    assert parse_device("b200") is None and parse_device("b200:3") == 3


def test_every_example_operator_is_registered():
    names = {k[0] for k in cuda.registered()}
    assert {"add_kernel", "softmax_kernel", "matmul_kernel", "dense_layer_kernel", "attn_fwd_kernel",
            "layernorm_kernel"} <= names
    for k in (add_kernel, softmax_kernel, matmul_kernel, dense_layer_kernel, attn_fwd_kernel):
        assert (k.__name__, tuple(k.arg_names)) in dict.fromkeys(cuda.registered())


def test_unregistered_kernel_raises_not_implemented():
    @triton.jit
    def my_kernel(x_ptr, n, BLOCK: tl.constexpr):
        pass

    with pytest.raises(NotImplementedError):
        cuda.run_on_b200(my_kernel, (1,), {"BLOCK": 4}, {"x_ptr": np.zeros(4, np.float32), "n": 4})


def test_extent():
    assert cuda.extent((3, 5), (4, 1)) == (0, 13)
    assert cuda.extent((3, -5), (4, 1)) == (-10, 3)
    assert cuda.extent((0, 5)) == (0, -1)


REF = os.environ.get("PITON_REFERENCE", "")


@pytest.mark.skipif(not (REF and os.path.isdir(os.path.join(REF, "examples"))),
                    reason="PITON_REFERENCE (a reference checkout) is not set")
def test_reference_jit_functions_match_the_registry():
    examples = os.path.join(REF, "examples")
    sys.path.insert(0, REF)
    sys.path.insert(0, examples)
    try:
        import kernels as ref_kernels
        import nn_kernels as ref_nn
    finally:
        sys.path.remove(examples)
        sys.path.remove(REF)
    reg = dict.fromkeys(cuda.registered())
    for k in (ref_kernels.add_kernel, ref_kernels.matmul_kernel, ref_kernels.softmax_kernel,
              ref_nn.dense_layer_kernel):
        assert (k.__name__, tuple(k.arg_names)) in reg
    # the reference's constexpr annotation is recognised by bind()
    x = np.zeros(4, np.float32)
    _, consts, _ = bind(ref_kernels.add_kernel.fn, (x, x, x, 4), dict(BLOCK_SIZE=4))
    assert consts == {"BLOCK_SIZE": 4}
