"""TinyGPT host side without a GPU: weight packing agrees with the kernel's layout
size, the float64 oracle is deterministic and produces in-vocabulary tokens."""

import numpy as np

from oracle import tinygpt_ref
from piton_b200 import tinygpt
from piton_b200.runtime.cuda._lib import lib


def test_packed_size_matches_the_kernel_layout():
    w = tinygpt.init_weights(0)
    assert tinygpt.pack(w).size == lib().piton_b200_tinygpt_weight_floats()
    assert abs(float(w["wte"].std()) - 0.02) < 2e-3


def test_oracle_decode_is_deterministic():
    w = tinygpt.init_weights(1)
    prompts = tinygpt.random_prompts(3, seed=2)
    a, la, na = tinygpt_ref.generate(w, prompts, 8)
    b, lb, nb = tinygpt_ref.generate(w, prompts, 8)
    assert a.shape == (3, 24) and np.array_equal(a, b) and np.array_equal(la, lb)
    assert a.min() >= 0 and a.max() < 65
    np.testing.assert_array_equal(a[:, :16], prompts)
