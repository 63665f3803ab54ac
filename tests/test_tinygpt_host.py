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


def test_host_model_decode_matches_reference_kernels_on_the_emulator():
    """The float64 host model against TinyGPT's greedy decode composed from the reference's own
    dense_layer_kernel, attn_fwd_kernel and layernorm_kernel on its emulator with a KV cache
    (tests/golden/make_golden.py case_tinygpt_decode): a 16-token prompt, 4 greedy steps.  The
    same tokens, and the logits that chose each of them within 2e-5."""
    import numpy as np

    from conftest import goldens
    from oracle import tinygpt_ref
    from piton_b200 import tinygpt
    gs = goldens("tinygpt_emu_decode_")
    assert gs
    for g in gs:
        w = tinygpt.init_weights(g.meta["weight_seed"])
        plen, new = g.meta["prompt_len"], g.meta["new_tokens"]
        toks, _, near = tinygpt_ref.generate(w, g["prompt"][None], new)
        assert near[0] < 0                                  # no near tie on this prompt
        np.testing.assert_array_equal(toks[0, plen:], g["tokens"])
        lg = tinygpt_ref.teacher_forced_logits(w, toks, plen)[0]
        np.testing.assert_allclose(lg, g["logits"], rtol=0, atol=2e-5)
